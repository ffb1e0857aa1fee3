"""The reference's split-search unit tests (src/training/split.rs:856-1110)
on the CPU oracle's component: known answers for the missing direction,
missing rows alone on one side, a constant feature, the default direction
when nothing is missing, and gains equal bit for bit to an independent
brute-force enumeration over random blocks (split.rs:802-898).  A case is a
column-major block of bins (missing = 255), gradients quantized by the
reference's quantizer, the histogram and the node sum in fixed point."""
import numpy as np
import pytest

MISSING = 255


class Case:
    def __init__(self, oracle, block, n_rows, feat_offsets, grads):
        self.o = oracle
        self.block = np.asarray(block, np.uint16).reshape(len(feat_offsets) - 1, n_rows)
        self.n = n_rows
        self.off = np.asarray(feat_offsets, np.uint32)
        g = np.asarray(grads, np.float32).reshape(-1, 2)
        self.scales = oracle.quantizer(g, n_rows)
        self.fixed, self.sum = oracle.to_fixed(g, self.scales)

    def f(self, pair):  # fixed point back to f64 (power-of-two scales: exact)
        return pair[0] / self.scales[0], pair[1] / self.scales[1]

    def best(self, **kw):
        miss = np.full(len(self.off) - 1, MISSING, np.uint16)
        h = self.o.hist(self.block, self.off, miss, self.fixed)
        params = dict(dict(reg_lambda=1.0, min_child_weight=0.0), **kw)
        r = self.o.best_split(h, self.off, self.sum, self.scales, **params)
        return r if r.found else None

    def partition(self, feat, bin_, missing_left):
        l, r = np.zeros(2, np.int64), np.zeros(2, np.int64)
        for row in range(self.n):
            b = int(self.block[feat, row])
            left = missing_left if b == MISSING else b < bin_
            if left:
                l = (l.astype(np.uint64) + self.fixed[row].astype(np.uint64)).astype(np.int64)
            else:
                r = (r.astype(np.uint64) + self.fixed[row].astype(np.uint64)).astype(np.int64)
        return l, r


def _pairs(gs, h=1.0):
    return [[g, h] for g in gs]


@pytest.mark.parametrize("missing_grad", [-1.0, 1.0])
def test_missing_goes_to_the_side_it_agrees_with(oracle, missing_grad):
    c = Case(oracle, [0, 0, 1, 1, MISSING, MISSING], 6, [0, 2], _pairs([-1, -1, 1, 1, missing_grad, missing_grad]))
    s = c.best()
    assert s.bin == 1
    if missing_grad < 0:
        assert s.missing_left and c.f((s.left_g, s.left_h))[0] == -4.0 and c.f((s.right_g, s.right_h))[0] == 2.0
    else:
        assert not s.missing_left and c.f((s.left_g, s.left_h))[0] == -2.0 and c.f((s.right_g, s.right_h))[0] == 4.0


def test_missing_alone_on_one_side_is_a_valid_split(oracle):
    c = Case(oracle, [0, 1, 0, 1, MISSING, MISSING], 6, [0, 2], _pairs([1, 1, 1, 1, -3, -3]))
    s = c.best()
    assert s.bin == 2 and not s.missing_left
    assert c.f((s.left_g, s.left_h))[0] == 4.0 and c.f((s.right_g, s.right_h))[0] == -6.0


def test_constant_feature_without_missing_has_no_split(oracle):
    c = Case(oracle, [0, 0, 0, 0], 4, [0, 1], _pairs([1, -1, 2, -2]))
    assert c.best() is None


def _random_case(oracle, seed, n_rows, n_feats, missing_pct):
    rng = np.random.default_rng(seed)
    n_bins = [2 + f % 5 for f in range(n_feats)]
    off = np.concatenate([[0], np.cumsum(n_bins)]).astype(np.uint32)
    block = np.zeros((n_feats, n_rows), np.uint16)
    for f in range(n_feats):
        block[f] = rng.integers(0, n_bins[f], n_rows)
        block[f][rng.integers(0, 100, n_rows) < missing_pct] = MISSING
    g = rng.uniform(-1, 1, n_rows).astype(np.float32)
    h = (0.05 + 0.2 * rng.integers(0, 1000, n_rows) / 1000.0).astype(np.float32)
    return Case(oracle, block.ravel(), n_rows, off, np.stack([g, h], 1))


def test_no_missing_means_default_direction_stays_right(oracle):
    for seed in range(10):
        s = _random_case(oracle, seed, 32, 3, 0).best()
        assert s is not None and not s.missing_left


def _side_gain(g, h, lam):
    """split.rs:187-197 xgb_weight and :216-223 gain_given_weight with alpha =
    0 and no max_delta_step: w = f32(-G/(H+lambda)); -(2 G w + (H+lambda) w*w)
    with the square taken in f32, the side's gain rounded to f32."""
    if h <= 0.0:
        return np.float32(0.0)
    w = np.float32(-g / (h + lam))
    sq = float(np.float32(w * w))
    return np.float32(-(2.0 * g * float(w) + (h + lam) * sq))


def _brute_force(c, lam, mcw, gamma=0.0):
    """split.rs:802-851 brute_force: partition the rows directly for every
    (feature, threshold, missing direction), skipping the histogram and the
    node-sum subtraction; the first strict maximum wins.  The gain is the one
    training evaluates: types.rs:637 ``uses_given_weight`` is always true, so
    every split goes through split.rs:234-252 (given-weight form, unbounded
    node: sides rounded to f32 and summed in f32, minus the f32 parent gain)
    and the validity rule of split.rs:241 (both Hessians > 0 and >=
    min_child_weight).  The reference's own brute force checks the
    ``monotone=None`` branch instead (G^2/(H+lambda) in f64, split.rs:89-93),
    which training never takes; ``_g2_form`` below restates it for the
    within-rounding comparison."""
    ng, nh = c.f(c.sum)
    parent = _side_gain(ng, nh, lam)
    best = None
    for feat in range(len(c.off) - 1):
        nb = int(c.off[feat + 1] - c.off[feat])
        for b in range(nb + 1):
            for ml in (False, True):
                l, r = c.partition(feat, b, ml)
                (lg, lh), (rg, rh) = c.f(l), c.f(r)
                if not (lh > 0.0 and rh > 0.0 and lh >= mcw and rh >= mcw):
                    continue
                loss = np.float32(np.float32(_side_gain(lg, lh, lam) + _side_gain(rg, rh, lam)) - parent)
                g = np.float32(float(loss) - gamma)
                if not g > np.float32(1e-6):
                    continue
                if best is None or g > best[0]:
                    best = (g, feat, b, ml, l, r)
    return best


def _g2_form(c, feat, b, ml, lam, gamma=0.0):
    """split.rs:89-93 split_gain: GL^2/(HL+lambda) + GR^2/(HR+lambda) -
    G^2/(H+lambda) - gamma in f64, rounded once to f32."""
    ng, nh = c.f(c.sum)
    l, r = c.partition(feat, b, ml)
    (lg, lh), (rg, rh) = c.f(l), c.f(r)
    return np.float32(lg * lg / (lh + lam) + rg * rg / (rh + lam) - ng * ng / (nh + lam) - gamma)


def test_matches_brute_force_on_random_cases(oracle):
    checked = 0
    for seed in range(20):
        for missing_pct in (0, 10, 50):
            c = _random_case(oracle, seed, 64, 4, missing_pct)
            lam, mcw = 1.0 + seed % 3, (seed % 4) * 0.5
            got = c.best(reg_lambda=lam, min_child_weight=mcw)
            want = _brute_force(c, lam, mcw)
            if want is None:
                assert got is None
                continue
            assert got is not None
            assert np.float32(got.gain).view(np.uint32) == want[0].view(np.uint32), (seed, missing_pct)
            # the two algebraically equal forms agree up to the f32 rounding of
            # the side and parent terms, which cancel in the difference
            g2 = _g2_form(c, got.feat, got.bin, bool(got.missing_left), lam)
            ng, nh = c.f(c.sum)
            scale = max(abs(float(_side_gain(ng, nh, lam))), abs(float(g2)), 1.0)
            assert abs(float(g2) - float(want[0])) <= 8 * np.spacing(np.float32(scale)), (seed, missing_pct)
            if (got.feat, got.bin, bool(got.missing_left)) == want[1:4]:
                assert (got.left_g, got.left_h) == tuple(want[4]) and (got.right_g, got.right_h) == tuple(want[5])
            checked += 1
    assert checked > 40
