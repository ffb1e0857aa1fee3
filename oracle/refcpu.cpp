// refcpu — CPU restatement of the FerrisBoost reference training and
// explanation engine (mdai001/FerrisBoost 0.1.1, Rust).
//
// TEST INFRASTRUCTURE ONLY: the correctness oracle and the timed CPU baseline.
// The product (ferrisboost_b200/libfbgpu.so) never links or calls this file.
//
// The reference is Rust and cannot be built in this image (no cargo/rustc, no
// network for its crates), so this file restates its algorithm in C++.  Every
// function cites the reference source it follows (paths relative to the
// reference project).  Floating-point expressions keep the reference's
// evaluation order; the file is compiled with -ffp-contract=off and without
// fast-math so that no operation is fused or reassociated, and `expf`/`logf`
// come from glibc exactly as Rust's f32::exp / f32::ln do on Linux.
//
// Parity is pinned by the XGBoost 3.4.1 golden margins the reference ships in
// tests/fixtures (tests/bit_exact_vs_xgboost.rs:213-554): 18 unweighted, 13
// weighted and 13 monotone cases, checked bit for bit by tests/test_oracle.py.
// The multiclass objectives have no golden vectors in the reference: their
// restatement (softmax gradients, class base margins, K trees per round) is
// pinned piecewise against independent statements (tests/test_multiclass_oracle.py)
// and otherwise reuses the pinned single-output tree builder.
#include "refcpu.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <queue>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

thread_local std::string g_err;
thread_local double g_setup_s = 0.0;
thread_local std::vector<double> g_round_s;

constexpr float kMinGainEps = 1e-6f;  // split.rs:15 MIN_GAIN_EPS
constexpr float kRtEps = 1e-6f;       // objective.rs:18 K_RT_EPS

struct GP { float g, h; };                 // types.rs:101 GradPair
struct FX { int64_t g, h; };               // types.rs:151 GradPairFixed

inline FX fx_add(FX a, FX b) {  // wrapping add, types.rs:204-217 (release)
    return {(int64_t)((uint64_t)a.g + (uint64_t)b.g), (int64_t)((uint64_t)a.h + (uint64_t)b.h)};
}
inline FX fx_sub(FX a, FX b) {
    return {(int64_t)((uint64_t)a.g - (uint64_t)b.g), (int64_t)((uint64_t)a.h - (uint64_t)b.h)};
}
inline bool fx_eq(FX a, FX b) { return a.g == b.g && a.h == b.h; }

// ---------------------------------------------------------------- quantizer
// types.rs:366-385 pow2_scale
double pow2_scale(double max_abs, uint64_t n_rows) {
    if (!(max_abs > 0.0) || !std::isfinite(max_abs)) return 1.0;
    double budget = (double)(1ull << 62) / (double)std::max<uint64_t>(n_rows, 1);
    double raw = budget / max_abs;
    if (!std::isfinite(raw) || raw <= 0.0) return 1.0;
    double l = std::floor(std::log2(raw));
    int k;
    if (l >= 2147483647.0) k = 2147483647;
    else if (l <= -2147483648.0) k = (int)-2147483647 - 1;
    else k = (int)l;
    k = std::min(1000, std::max(-1000, k));
    return std::ldexp(1.0, k);
}

struct Quantizer {  // types.rs:239-340 GradQuantizer
    double gs = 1, hs = 1, gi = 1, hi = 1;
    static Quantizer from_scales(double gs, double hs) {
        Quantizer q; q.gs = gs; q.hs = hs; q.gi = 1.0 / gs; q.hi = 1.0 / hs; return q;
    }
    FX to_fixed(GP v) const {  // types.rs:334-337 quantize
        return {(int64_t)std::round((double)v.g * gs), (int64_t)std::round((double)v.h * hs)};
    }
    void to_f64(FX v, double& g, double& h) const {  // types.rs:298-310
        g = (double)v.g * gi;
        h = (double)v.h * hi;
    }
    float hess_f32(FX v) const { return (float)((double)v.h * hi); }
};

inline double finite_abs(float v) {  // types.rs:325-331
    return std::isfinite(v) ? std::fabs((double)v) : std::numeric_limits<double>::infinity();
}

// ---------------------------------------------------------------- sketch
// data/sketch.rs: log-structured weighted quantile sketch.
struct Entry { float value, weight, rmin, rmax; float rmid() const { return 0.5f * (rmin + rmax); } };

std::vector<Entry> build_summary(std::vector<std::pair<float, float>>& pairs) {  // sketch.rs:305-329
    std::sort(pairs.begin(), pairs.end(),
              [](const std::pair<float, float>& a, const std::pair<float, float>& b) { return a.first < b.first; });
    std::vector<Entry> out;
    out.reserve(pairs.size());
    float acc = 0.0f;
    size_t i = 0;
    while (i < pairs.size()) {
        float v = pairs[i].first;
        float w = 0.0f;
        while (i < pairs.size() && pairs[i].first == v) { w += pairs[i].second; i++; }
        out.push_back({v, w, acc, acc + w});
        acc += w;
    }
    return out;
}

std::vector<Entry> dedup_same_value(const std::vector<Entry>& e) {  // sketch.rs:378-392
    std::vector<Entry> out;
    out.reserve(e.size());
    for (const Entry& x : e) {
        if (!out.empty() && out.back().value == x.value) {
            Entry& l = out.back();
            l.weight += x.weight;
            l.rmin = std::min(l.rmin, x.rmin);
            l.rmax = std::max(l.rmax, x.rmax);
        } else {
            out.push_back(x);
        }
    }
    return out;
}

std::vector<Entry> merge_entries(const std::vector<Entry>& a, const std::vector<Entry>& b) {  // sketch.rs:336-376
    if (a.empty()) return b;
    if (b.empty()) return a;
    std::vector<Entry> out;
    out.reserve(a.size() + b.size());
    size_t i = 0, j = 0;
    float pass_a = 0.0f, pass_b = 0.0f;
    while (i < a.size() || j < b.size()) {
        bool take_a;
        if (i < a.size() && j < b.size()) take_a = a[i].value <= b[j].value;
        else take_a = i < a.size();
        if (take_a) {
            Entry e = a[i];
            out.push_back({e.value, e.weight, e.rmin + pass_b, e.rmax + pass_b});
            pass_a = e.rmax;
            i++;
        } else {
            Entry e = b[j];
            out.push_back({e.value, e.weight, e.rmin + pass_a, e.rmax + pass_a});
            pass_b = e.rmax;
            j++;
        }
    }
    return dedup_same_value(out);
}

std::vector<Entry> compress(const std::vector<Entry>& e, size_t max_size) {  // sketch.rs:403-435
    size_t n = e.size();
    if (n <= max_size) return e;
    float total = e[n - 1].rmax;
    size_t slots = max_size - 1;
    std::vector<Entry> out;
    out.reserve(max_size);
    out.push_back(e[0]);
    size_t taken = 0;
    for (size_t k = 1; k < slots; k++) {
        float target = total * (float)k / (float)slots;
        size_t j = taken + 1;
        while (j < n - 1 && e[j].rmid() < target) j++;
        size_t ceiling = n - 1 - (slots - 1 - k);
        j = std::min(std::max(j, taken + 1), ceiling);
        if (j > taken) { out.push_back(e[j]); taken = j; }
    }
    if (taken < n - 1) out.push_back(e[n - 1]);
    return out;
}

float midpoint(float a, float b) {  // sketch.rs:290-302
    float d = b - a;
    float m = std::isfinite(d) ? a + d * 0.5f : a * 0.5f + b * 0.5f;
    return m <= a ? b : m;
}

struct FeatureSketch {  // sketch.rs:49-281
    std::vector<std::pair<float, float>> buffer;
    std::vector<std::vector<Entry>> levels;
    std::vector<bool> occupied;
    size_t limit;
    explicit FeatureSketch(size_t max_bins) : limit(std::max<size_t>(max_bins * 16, 32)) { buffer.reserve(limit); }
    void push(float v, float w) {  // sketch.rs:128-147
        if (std::isnan(v) || w <= 0.0f) return;
        buffer.push_back({v, w});
        if (buffer.size() >= limit) drain();
    }
    void drain() {  // sketch.rs:149-158
        if (buffer.empty()) return;
        std::vector<Entry> s = compress(build_summary(buffer), limit);
        buffer.clear();
        insert_level(std::move(s));
    }
    void insert_level(std::vector<Entry> cur) {  // sketch.rs:161-180
        size_t lvl = 0;
        for (;;) {
            if (lvl == levels.size()) { levels.push_back(std::move(cur)); occupied.push_back(true); return; }
            if (!occupied[lvl]) { levels[lvl] = std::move(cur); occupied[lvl] = true; return; }
            std::vector<Entry> existing = std::move(levels[lvl]);
            occupied[lvl] = false;
            levels[lvl].clear();
            cur = compress(merge_entries(existing, cur), limit);
            lvl++;
        }
    }
    std::vector<Entry> collapse() {  // sketch.rs:183-201
        drain();
        std::vector<Entry> acc;
        for (size_t l = 0; l < levels.size(); l++) {
            if (!occupied[l]) continue;
            acc = acc.empty() ? levels[l] : merge_entries(acc, levels[l]);
        }
        levels.clear(); occupied.clear();
        if (!acc.empty()) { levels.push_back(compress(acc, limit)); occupied.push_back(true); }
        return levels.empty() ? std::vector<Entry>() : levels[0];
    }
    std::vector<float> cuts(size_t max_bins) {  // sketch.rs:236-275
        size_t n_cuts = max_bins >= 1 ? max_bins - 1 : 0;
        if (n_cuts == 0) return {};
        std::vector<Entry> e = collapse();
        if (e.empty()) return {};
        std::vector<float> out;
        if (e.size() <= n_cuts) {
            for (size_t i = 0; i + 1 < e.size(); i++) out.push_back(midpoint(e[i].value, e[i + 1].value));
            return out;
        }
        float total = e.back().rmax;
        for (size_t k = 1; k <= n_cuts; k++) {
            float target = total * (float)k / (float)max_bins;
            size_t idx = std::partition_point(e.begin(), e.end(), [&](const Entry& x) { return x.rmid() < target; }) - e.begin();
            idx = std::min(idx, e.size() - 1);
            float v = e[idx].value;
            if (out.empty() || v > out.back()) out.push_back(v);
        }
        return out;
    }
};

// ---------------------------------------------------------------- cuts / bins
struct Cuts {  // data/columns.rs:54-342
    std::vector<float> values;
    std::vector<uint32_t> offsets;  // F+1
    std::vector<uint8_t> cat;       // per feature
    uint32_t n_feats() const { return (uint32_t)offsets.size() - 1; }
    uint32_t n_cuts(uint32_t f) const { return offsets[f + 1] - offsets[f]; }
    uint32_t n_bins(uint32_t f) const { return n_cuts(f) + 1; }
    bool is_cat(uint32_t f) const { return !cat.empty() && cat[f]; }
    // bins.rs:58-66 BinWidth::for_feature: 8-bit unless more bins are needed.
    bool wide(uint32_t f) const {
        uint32_t nb = n_bins(f);
        return is_cat(f) ? nb > 254u : nb > 255u;
    }
    uint16_t missing(uint32_t f) const { return wide(f) ? 65535 : 255; }
    uint32_t find_bin(uint32_t f, float v) const {  // columns.rs:335-341
        if (is_cat(f)) {  // categorical.rs:360-370 code_to_bin
            uint32_t nb = n_bins(f);
            if (v >= 0.0f && v < (float)nb) return (uint32_t)v;
            return missing(f) - 1u;
        }
        const float* c = values.data() + offsets[f];
        const float* e = c + n_cuts(f);
        return (uint32_t)(std::upper_bound(c, e, v) - c);
    }
    float threshold(uint32_t f, uint32_t bin) const {  // tree.rs:991-1000 split_threshold
        uint32_t nc = n_cuts(f);
        if (bin == 0) return -std::numeric_limits<float>::max();
        if (bin > nc) return std::numeric_limits<float>::max();
        return values[offsets[f] + bin - 1];
    }
};

int n_threads(int32_t nthread) {
#ifdef _OPENMP
    return nthread > 0 ? nthread : omp_get_max_threads();
#else
    (void)nthread;
    return 1;
#endif
}

// source/dense.rs:136-208: one sketch per feature built serially from all
// rows (no cross-thread merge, so the cuts do not depend on the thread count).
Cuts sketch_cuts(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                 const uint8_t* categorical, int nth) {
    std::vector<std::vector<float>> per(F);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
    for (int64_t f = 0; f < (int64_t)F; f++) {
        if (categorical && categorical[f]) {  // sketch.rs:128-136 categorical scan
            int32_t max_code = -1;
            for (uint64_t r = 0; r < n; r++) {
                float v = X[r * F + f];
                if (std::isnan(v)) continue;
                // categorical.rs:264-266 invalid_code; an invalid code is an input error
                if (v < 0.0f || v > 65533.0f || v != std::trunc(v)) throw std::runtime_error("invalid categorical code");
                max_code = std::max(max_code, (int32_t)v);
            }
            std::vector<float> c;
            for (int32_t k = 1; k <= std::max(max_code, 0); k++) c.push_back((float)k);  // columns.rs:127-129
            per[f] = c;
            continue;
        }
        FeatureSketch sk(max_bin);
        for (uint64_t r = 0; r < n; r++) sk.push(X[r * F + f], w ? w[r] : 1.0f);
        per[f] = sk.cuts(max_bin);
    }
    Cuts c;
    c.offsets.push_back(0);
    for (uint32_t f = 0; f < F; f++) {
        c.values.insert(c.values.end(), per[f].begin(), per[f].end());
        c.offsets.push_back((uint32_t)c.values.size());
    }
    if (categorical) c.cat.assign(categorical, categorical + F);
    return c;
}

// Column-major bin codes (dense.rs:288-308 quantize_dense).
void quantize_cols(const float* X, uint64_t n, uint32_t F, const Cuts& c, std::vector<uint16_t>& out, int nth) {
    out.resize((size_t)F * n);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
    for (int64_t f = 0; f < (int64_t)F; f++) {
        uint16_t miss = c.missing((uint32_t)f);
        uint16_t* dst = out.data() + (size_t)f * n;
        for (uint64_t r = 0; r < n; r++) {
            float v = X[r * F + f];
            dst[r] = std::isnan(v) ? miss : (uint16_t)c.find_bin((uint32_t)f, v);
        }
    }
}

// ---------------------------------------------------------------- params
struct Params {
    rc_params p;
    std::vector<int8_t> mono;
    std::vector<uint8_t> cat;
    int8_t mono_of(uint32_t f) const { return f < mono.size() ? mono[f] : 0; }
};

// ---------------------------------------------------------------- split
// training/split.rs
struct Bounds { float lower, upper; };  // split.rs:113-155 NodeBounds
const Bounds kUnbounded{-std::numeric_limits<float>::max(), std::numeric_limits<float>::max()};
inline float bounds_apply(Bounds b, float w) { return w < b.lower ? b.lower : (w > b.upper ? b.upper : w); }

double threshold_l1(double g, float alpha) {  // split.rs:171-181
    double a = (double)alpha;
    if (g > a) return g - a;
    if (g < -a) return g + a;
    return 0.0;
}
float xgb_weight(double g, double h, const rc_params& p) {  // split.rs:187-197
    if (h <= 0.0) return 0.0f;
    double dw = -threshold_l1(g, p.alpha) / (h + (double)p.lambda);
    float mds = p.max_delta_step;
    if (mds != 0.0f && std::fabs(dw) > (double)mds) dw = std::copysign((double)mds, dw);
    return (float)dw;
}
float gain_given_weight(double g, double h, float w, const rc_params& p) {  // split.rs:216-223
    if (h <= 0.0) return 0.0f;
    double square = (double)(w * w);
    double l1 = 2.0 * (double)p.alpha * (double)std::fabs(w);
    return (float)(-((2.0 * g * (double)w + (h + (double)p.lambda) * square) + l1));
}
float bounded_node_gain(double g, double h, const rc_params& p, Bounds b) {  // split.rs:226-229
    float w = bounds_apply(b, xgb_weight(g, h, p));
    return gain_given_weight(g, h, w, p);
}
// split.rs:234-252 bounded_split_gain; returns false when the candidate is invalid.
bool bounded_split_gain(float parent, double lg, double lh, double rg, double rh, int8_t constraint,
                        Bounds b, const rc_params& p, float& out) {
    double mcw = (double)p.min_child_weight;
    if (!(lh > 0.0 && rh > 0.0 && lh >= mcw && rh >= mcw)) return false;
    float wl = bounds_apply(b, xgb_weight(lg, lh, p));
    float wr = bounds_apply(b, xgb_weight(rg, rh, p));
    if ((constraint > 0 && wl > wr) || (constraint < 0 && wl < wr)) return false;
    float gain = gain_given_weight(lg, lh, wl, p) + gain_given_weight(rg, rh, wr, p);
    float loss = gain - parent;
    out = (float)((double)loss - (double)p.gamma);
    return true;
}

struct Cand {  // split.rs:17-52 SplitCandidate
    bool found = false;
    uint32_t feat = 0, bin = 0;
    float gain = 0;
    FX left{0, 0}, right{0, 0};
    bool missing_left = false;
    bool is_cat = false;
    std::vector<uint32_t> cats;  // right-going set, 32-bit words
};

inline void update_best(Cand& best, const Cand& c) {  // split.rs:260-270
    if (!(c.gain > kMinGainEps)) return;
    if (!best.found || c.gain > best.gain) best = c;
}

// split.rs:484-617 enumerate_categorical (XGBoost EnumerateOneHot / EnumeratePart)
void enumerate_categorical(uint32_t feat, const FX* bins, uint32_t n, FX node_sum, const Quantizer& q,
                           const Params& P, float parent, Bounds b, Cand& best) {
    const rc_params& p = P.p;
    int8_t cons = P.mono_of(feat);
    struct Local { float gain; FX left, right; bool ml; size_t at; };
    bool have = false;
    Local loc{};
    auto consider = [&](FX left, FX right, bool ml, size_t at) {
        double lg, lh, rg, rh;
        q.to_f64(left, lg, lh);
        q.to_f64(right, rg, rh);
        float gain;
        if (!bounded_split_gain(parent, lg, lh, rg, rh, cons, b, p, gain)) return;
        if (gain > kMinGainEps && (!have || gain > loc.gain)) { loc = {gain, left, right, ml, at}; have = true; }
    };
    auto words_for = [&](const std::vector<uint32_t>& members) {
        std::vector<uint32_t> w((n + 31) / 32, 0);
        for (uint32_t c : members) w[c / 32] |= 1u << (c % 32);
        while (!w.empty() && w.back() == 0) w.pop_back();
        return w;
    };
    auto finish = [&](const std::vector<uint32_t>& members) {
        if (!have) return;
        Cand c;
        c.found = true; c.feat = feat; c.bin = 0; c.gain = loc.gain; c.left = loc.left; c.right = loc.right;
        c.missing_left = loc.ml; c.is_cat = true; c.cats = words_for(members);
        update_best(best, c);
    };
    if ((uint64_t)n < (uint64_t)p.max_cat_to_onehot) {
        FX fsum{0, 0};
        for (uint32_t i = 0; i < n; i++) fsum = fx_add(fsum, bins[i]);
        FX missing = fx_sub(node_sum, fsum);
        for (uint32_t i = 0; i < n; i++) {
            consider(fx_sub(node_sum, bins[i]), bins[i], true, i);
            FX right = fx_add(bins[i], missing);
            consider(fx_sub(node_sum, right), right, false, i);
        }
        if (have) finish({(uint32_t)loc.at});
        return;
    }
    std::vector<float> weights(n);
    for (uint32_t i = 0; i < n; i++) {
        double g, h;
        q.to_f64(bins[i], g, h);
        weights[i] = xgb_weight(g, h, p);
    }
    std::vector<uint32_t> order(n);
    for (uint32_t i = 0; i < n; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t c) { return weights[a] < weights[c]; });
    size_t n_scan = std::min<size_t>(p.max_cat_threshold, n);
    if (n_scan < 2) return;
    auto prefix = [&](size_t k) { return std::vector<uint32_t>(order.begin(), order.begin() + k); };
    FX right{0, 0};
    for (size_t k = 0; k + 1 < n_scan; k++) {
        right = fx_add(right, bins[order[k]]);
        consider(fx_sub(node_sum, right), right, true, k + 1);
    }
    if (have) { finish(prefix(loc.at)); have = false; }
    FX left{0, 0};
    for (size_t j = n; j-- > n - (n_scan - 1);) {
        left = fx_add(left, bins[order[j]]);
        consider(left, fx_sub(node_sum, left), false, j);
    }
    if (have) finish(prefix(loc.at));
}

// split.rs:331-461 best_split_in_block_typed, always in the given-weight form
// (types.rs:628-639 uses_given_weight() == true; training/mod.rs:5000-5005).
// Features are enumerated in ascending global order, which together with the
// strict-greater rule equals the cross-block reduce_best (split.rs:631-642).
Cand best_split(const FX* hist, uint32_t F, const uint32_t* off, FX node_sum, const Quantizer& q, const Params& P,
                Bounds b, const uint8_t* enabled) {
    const rc_params& p = P.p;
    double ng, nh;
    q.to_f64(node_sum, ng, nh);
    float parent = bounded_node_gain(ng, nh, p, b);
    Cand best;
    for (uint32_t f = 0; f < F; f++) {
        if (enabled && !enabled[f]) continue;
        const FX* bins = hist + off[f];
        uint32_t nb = off[f + 1] - off[f];
        if (!P.cat.empty() && P.cat[f]) {
            enumerate_categorical(f, bins, nb, node_sum, q, P, parent, b, best);
            continue;
        }
        int8_t cons = P.mono_of(f);
        FX left{0, 0};
        for (uint32_t i = 0; i < nb; i++) {
            left = fx_add(left, bins[i]);
            FX right = fx_sub(node_sum, left);
            double lg, lh, rg, rh;
            q.to_f64(left, lg, lh);
            q.to_f64(right, rg, rh);
            float gain;
            if (!bounded_split_gain(parent, lg, lh, rg, rh, cons, b, p, gain)) continue;
            if (!(gain > kMinGainEps)) continue;
            if (!best.found || gain > best.gain) {
                best.found = true; best.feat = f; best.bin = i + 1; best.gain = gain;
                best.left = left; best.right = right; best.missing_left = false; best.is_cat = false; best.cats.clear();
            }
        }
        if (fx_eq(left, node_sum)) continue;
        FX right{0, 0};
        for (uint32_t i = nb; i-- > 0;) {
            right = fx_add(right, bins[i]);
            FX l = fx_sub(node_sum, right);
            double lg, lh, rg, rh;
            q.to_f64(l, lg, lh);
            q.to_f64(right, rg, rh);
            float gain;
            if (!bounded_split_gain(parent, lg, lh, rg, rh, cons, b, p, gain)) continue;
            if (!(gain > kMinGainEps)) continue;
            if (!best.found || gain > best.gain) {
                best.found = true; best.feat = f; best.bin = i; best.gain = gain;
                best.left = l; best.right = right; best.missing_left = true; best.is_cat = false; best.cats.clear();
            }
        }
    }
    return best;
}

// ---------------------------------------------------------------- tree
struct Node {  // model/tree.rs:52-79
    uint32_t feat = 0;
    float cond = 0;
    int32_t left = -1, right = -1;
    bool default_left = false;
    float leaf = 0;
    bool is_leaf = true;
    float gain = 0;
    float hess = 0;
    bool is_cat = false;
    std::vector<uint32_t> cats;  // right-going set, 32-bit words
};
struct Tree {
    std::vector<Node> nodes;
    int push_leaf(float v, float h) { Node n; n.leaf = v; n.hess = h; nodes.push_back(n); return (int)nodes.size() - 1; }
    void split_leaf(int node, uint32_t feat, float cond, bool dl, float gain, float lv, float lh, float rv, float rh,
                    int& l, int& r) {  // tree.rs:140-170
        l = push_leaf(lv, lh);
        r = push_leaf(rv, rh);
        Node& n = nodes[node];
        n.feat = feat; n.cond = cond; n.left = l; n.right = r; n.default_left = dl; n.leaf = 0.0f;
        n.is_leaf = false; n.gain = gain;
    }
};

bool cat_goes_left(const std::vector<uint32_t>& words, float v) {  // categorical.rs:330-345
    if (std::isnan(v)) return false;
    if (v < 0.0f || v >= 16777216.0f) return true;
    uint32_t c = (uint32_t)v;
    if (c / 32 >= words.size()) return true;
    return ((words[c / 32] >> (c % 32)) & 1u) == 0;
}
inline bool node_goes_left(const Node& n, float v) {  // tree.rs:84-96
    if (std::isnan(v)) return n.default_left;
    if (n.is_cat) return cat_goes_left(n.cats, v);
    return v < n.cond;
}
float tree_leaf_value(const Tree& t, const float* x) {  // tree.rs:193-212
    if (t.nodes.empty()) return 0.0f;
    size_t i = 0;
    for (;;) {
        const Node& n = t.nodes[i];
        if (n.is_leaf) return n.leaf;
        i = node_goes_left(n, x[n.feat]) ? (size_t)n.left : (size_t)n.right;
    }
}

struct Model {
    std::vector<Tree> trees;
    float base_score = 0.5f;
    int objective = 1;
    std::vector<float> class_margins;  // multiclass: one base margin per class (tree.rs:260)
    uint32_t n_features = 0;
    float scale_pos_weight = 1.0f;
    std::vector<uint8_t> feature_types;
};

float base_margin(int objective, float base_score) {  // objective.rs:368-399
    if (objective == 1) {
        float x = std::min(std::max(base_score, kRtEps), 1.0f - kRtEps);
        return -std::log(1.0f / x - 1.0f);
    }
    return base_score;
}

// ---------------------------------------------------------------- gradients
// objective.rs:37-39 sigmoid; objective.rs:519-526 logistic; :513-516 squared error
inline GP gradient_of(float pred, float label, int objective) {
    if (objective == 1) {
        float s = 1.0f / (1.0f + std::exp(-pred));
        float h = s * (1.0f - s);
        return {s - label, h < 1e-16f ? 1e-16f : h};
    }
    return {pred - label, 1.0f};
}

// objective.rs:1175-1219 softmax_gradients of one row: wmax starts at the
// smallest positive normal f32 (XGBoost's numeric_limits<float>::min()),
// the exps are summed in f64, p = exp / (f32)sum, h = max(2 p (1 - p) w, 1e-16)
// and the label's class takes p - 1; g = p w.
inline void softmax_row(const float* m, uint32_t K, float label, float wt, GP* out) {
    float wmax = std::numeric_limits<float>::min();
    for (uint32_t k = 0; k < K; k++) wmax = std::fmax(m[k], wmax);
    double wsum = 0.0;
    for (uint32_t k = 0; k < K; k++) wsum += (double)std::exp(m[k] - wmax);
    for (uint32_t k = 0; k < K; k++) {
        float p = std::exp(m[k] - wmax) / (float)wsum;
        const float h = std::fmax(2.0f * p * (1.0f - p) * wt, 1e-16f);
        if (label == (float)k) p -= 1.0f;
        out[k] = {p * wt, h};
    }
}

// objective.rs:1225-1247 initial_class_margins (XGBoost SoftmaxMultiClassObj
// InitEstimation): weighted class frequencies counted in f32 in row order,
// log(freq + kRtEps), minus their mean (0 + v0/K + v1/K + ... in f32).
std::vector<float> initial_class_margins(const float* y, uint64_t n, const float* w, uint32_t K) {
    std::vector<float> bins(K, 0.0f);
    for (uint64_t i = 0; i < n; i++) bins[(size_t)y[i]] += w ? w[i] : 1.0f;
    double sum_w = (double)n;
    if (w) {
        sum_w = 0.0;
        for (uint64_t i = 0; i < n; i++) sum_w += (double)w[i];
    }
    if (sum_w < (double)kRtEps) return std::vector<float>(K, 0.0f);
    const double inv = 1.0 / sum_w;
    std::vector<float> logs(K);
    for (uint32_t k = 0; k < K; k++) logs[k] = std::log((float)((double)bins[k] * inv) + kRtEps);
    const float nk = (float)K;
    float mean = 0.0f;
    for (uint32_t k = 0; k < K; k++) mean = mean + logs[k] / nk;
    for (uint32_t k = 0; k < K; k++) logs[k] = logs[k] - mean;
    return logs;
}

// objective.rs:41-61 label_mean; objective.rs:403-474 initial_base_score
float estimate_base_score(const float* y, uint64_t n, const float* w) {
    if (!w) {
        double nn = (double)n, acc = 0.0;
        for (uint64_t i = 0; i < n; i++) acc = acc + (double)y[i] / nn;
        return (float)acc;
    }
    double sw = 0.0;
    for (uint64_t i = 0; i < n; i++) sw = sw + (double)w[i];
    if (sw <= 0.0) return 0.5f;
    double acc = 0.0;
    for (uint64_t i = 0; i < n; i++) acc = acc + (double)y[i] / sw * (double)w[i];
    return (float)acc;
}

// objective.rs:403-493 initial_base_score for squared error and logistic:
// with |scale_pos_weight - 1| > 1e-6 (f32) one Newton step from margin 0 over
// the gradient weights (XGBoost FitIntercept; objective.rs:480-493
// newton_base_score), else the label mean.  Per row the pair at margin 0 is
// weighted in f32 and summed in f64; the step -G / max(H, 1e-6f) is rounded to
// f32 and mapped through the objective's transform (sigmoid, objective.rs:37).
float initial_base_score(int objective, const float* y, uint64_t n, const float* w, const float* gw, float spw) {
    if (!(std::fabs(spw - 1.0f) > 1e-6f)) return estimate_base_score(y, n, w);
    double sg = 0.0, sh = 0.0;
    const float s0 = 1.0f / (1.0f + std::exp(-0.0f));
    for (uint64_t i = 0; i < n; i++) {
        float g = objective == 1 ? s0 - y[i] : 0.0f - y[i];
        float h = objective == 1 ? std::max(s0 * (1.0f - s0), 1e-16f) : 1.0f;
        if (gw) { g = g * gw[i]; h = h * gw[i]; }
        sg = sg + (double)g;
        sh = sh + (double)h;
    }
    const float m = (float)(-sg / std::max(sh, (double)1e-6f));
    return objective == 1 ? 1.0f / (1.0f + std::exp(-m)) : m;
}

// data/subsample.rs:45-78
inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
inline uint64_t row_hash(uint64_t row, uint64_t seed, uint64_t tree) {
    return mix64(seed ^ rotl(tree * 0x9E3779B97F4A7C15ull, 23) ^ (row * 0xD6E8FEB86659FD93ull));
}
uint64_t threshold_for(float rate) {
    if (rate >= 1.0f) return UINT64_MAX;
    if (!(rate > 0.0f)) return UINT64_MAX;
    return (uint64_t)((double)rate * (double)(1ull << 53));
}

// data/colsample.rs:29-104 SplitMix64 + Fisher-Yates per tree
struct SplitMix { uint64_t s; uint64_t next() { s += 0x9E3779B97F4A7C15ull; return mix64(s); }
    uint64_t below(uint64_t n) { uint64_t zone = UINT64_MAX - (UINT64_MAX % n) - 1; for (;;) { uint64_t v = next(); if (v <= zone) return v % n; } } };
uint32_t sampled_count(uint32_t nf, float rate) {
    if (nf == 0) return 0;
    double v = std::floor((double)rate * (double)nf);
    uint64_t c = (std::isfinite(v) && v >= 1.0) ? (uint64_t)v : 1;
    return (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(c, nf));
}
std::vector<uint32_t> sample_features(uint32_t nf, float rate, uint64_t seed, uint64_t round) {
    uint32_t take = sampled_count(nf, rate);
    std::vector<uint32_t> ids(nf);
    for (uint32_t i = 0; i < nf; i++) ids[i] = i;
    if (take >= nf) return ids;
    SplitMix rng{seed ^ rotl(round * 0x9E3779B97F4A7C15ull, 17)};
    for (uint32_t i = nf - 1; i >= 1; i--) {
        uint32_t j = (uint32_t)rng.below((uint64_t)i + 1);
        std::swap(ids[i], ids[j]);
    }
    ids.resize(take);
    std::sort(ids.begin(), ids.end());
    return ids;
}

// ---------------------------------------------------------------- histogram
// training/hist.rs:94-274.  Fixed-point accumulation is order independent, so
// the loop structure (features of one block per thread, rows tiled) only
// decides speed, never the integers.
void hist_nodes(const std::vector<uint16_t>& bins, uint64_t n, const Cuts& cuts, const std::vector<uint32_t>& hoff,
                const std::vector<FX>& gpair, const std::vector<const uint32_t*>& rows,
                const std::vector<size_t>& lens, std::vector<FX*>& outs, int nth) {
    uint32_t F = cuts.n_feats();
    const size_t kTile = 4096;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
    for (int64_t f = 0; f < (int64_t)F; f++) {
        const uint16_t* col = bins.data() + (size_t)f * n;
        uint16_t miss = cuts.missing((uint32_t)f);
        for (size_t k = 0; k < rows.size(); k++) {
            FX* h = outs[k] + hoff[f];
            const uint32_t* r = rows[k];
            size_t len = lens[k];
            for (size_t a = 0; a < len; a += kTile) {
                size_t e = std::min(len, a + kTile);
                for (size_t i = a; i < e; i++) {
                    uint32_t row = r[i];
                    uint16_t b = col[row];
                    if (b == miss) continue;
                    h[b] = fx_add(h[b], gpair[row]);
                }
            }
        }
    }
}

// training/mod.rs:5169-5207 fill_partition_bits: per-row direction.
inline bool row_goes_left(const uint16_t* col, uint32_t row, uint16_t miss, const Cand& c) {
    uint16_t b = col[row];
    if (b == miss) return c.missing_left;
    if (c.is_cat) {  // categorical set goes right
        uint32_t w = b / 32;
        bool in = w < c.cats.size() && ((c.cats[w] >> (b % 32)) & 1u);
        return !in;
    }
    return (uint32_t)b < c.bin;
}

// Stable partition of a node's rows into [left | right] (training/mod.rs:5231-5429).
size_t partition_rows(const uint32_t* in, size_t len, uint32_t* out, const uint16_t* col, uint16_t miss, const Cand& c) {
    size_t nl = 0;
    for (size_t i = 0; i < len; i++) if (row_goes_left(col, in[i], miss, c)) nl++;
    size_t a = 0, b = nl;
    for (size_t i = 0; i < len; i++) {
        if (row_goes_left(col, in[i], miss, c)) out[a++] = in[i];
        else out[b++] = in[i];
    }
    return nl;
}

struct Ctx {
    const Params& P;
    const Cuts& cuts;
    const std::vector<uint16_t>& bins;
    uint64_t n;
    std::vector<uint32_t> hoff;
    uint32_t total_bins;
    int nth;
};

// training/mod.rs:5069-5093 child_leaves (given-weight form)
void child_values(const Cand& c, const Quantizer& q, const rc_params& p, Bounds parent, int8_t cons, float& lv,
                  float& rv, Bounds& lb, Bounds& rb) {
    double g, h;
    q.to_f64(c.left, g, h);
    float wl = bounds_apply(parent, xgb_weight(g, h, p));
    q.to_f64(c.right, g, h);
    float wr = bounds_apply(parent, xgb_weight(g, h, p));
    float mid = (wl + wr) / 2.0f;  // split.rs:140-153 NodeBounds::children
    lb = parent; rb = parent;
    if (cons < 0) { lb.lower = mid; rb.upper = mid; }
    else if (cons > 0) { lb.upper = mid; rb.lower = mid; }
    lv = wl * p.eta;
    rv = wr * p.eta;
}

float leaf_of(FX sum, const Quantizer& q, const rc_params& p) {  // training/mod.rs:5096-5099
    double g, h;
    q.to_f64(sum, g, h);
    return xgb_weight(g, h, p) * p.eta;
}

struct LevelNode {  // training/mod.rs:3239-3251
    int node;
    size_t start, len;  // span in the current row buffer
    FX sum;
    int hist_from;      // -1 accumulate, else parent slot
    int sibling;        // slot in this level
    Bounds bounds;
};

// training/mod.rs:3357-4564 build_tree, depthwise policy, CPU backend.
Tree build_tree_depthwise(Ctx& C, const std::vector<FX>& gpair, FX root_sum, const Quantizer& q,
                          std::vector<float>& preds, const uint8_t* enabled) {
    const rc_params& p = C.P.p;
    Tree t;
    int root = t.push_leaf(leaf_of(root_sum, q, p), q.hess_f32(root_sum));
    std::vector<uint32_t> cur(C.n), nxt(C.n);
    for (uint64_t i = 0; i < C.n; i++) cur[i] = (uint32_t)i;
    std::vector<LevelNode> level{{root, 0, (size_t)C.n, root_sum, -1, -1, kUnbounded}};
    std::vector<std::vector<FX>> parent_hists;
    uint32_t leaf_count = 1;
    for (uint32_t depth = 0; depth < p.max_depth; depth++) {
        if (level.empty() || (p.max_leaves != 0 && leaf_count >= p.max_leaves)) break;
        // histograms: accumulate the smaller children, subtract the larger
        std::vector<std::vector<FX>> hists(level.size());
        std::vector<const uint32_t*> rows;
        std::vector<size_t> lens;
        std::vector<FX*> outs;
        for (size_t i = 0; i < level.size(); i++) {
            if (level[i].hist_from < 0) {
                hists[i].assign(C.total_bins, FX{0, 0});
                rows.push_back(cur.data() + level[i].start);
                lens.push_back(level[i].len);
                outs.push_back(hists[i].data());
            }
        }
        hist_nodes(C.bins, C.n, C.cuts, C.hoff, gpair, rows, lens, outs, C.nth);
        for (size_t i = 0; i < level.size(); i++) {
            if (level[i].hist_from >= 0) {
                std::vector<FX>& ph = parent_hists[level[i].hist_from];
                const std::vector<FX>& sib = hists[level[i].sibling];
                for (uint32_t k = 0; k < C.total_bins; k++) ph[k] = fx_sub(ph[k], sib[k]);
                hists[i] = std::move(ph);
            }
        }
        std::vector<Cand> chosen(level.size());
#pragma omp parallel for schedule(dynamic, 1) num_threads(C.nth)
        for (int64_t i = 0; i < (int64_t)level.size(); i++)
            chosen[i] = best_split(hists[i].data(), C.cuts.n_feats(), C.hoff.data(), level[i].sum, q, C.P,
                                   level[i].bounds, enabled);
        if (p.max_leaves != 0) {  // training/mod.rs:4140-4151
            uint32_t remaining = p.max_leaves > leaf_count ? p.max_leaves - leaf_count : 0;
            for (Cand& c : chosen) {
                if (!c.found) continue;
                if (remaining == 0) c.found = false; else remaining--;
            }
        }
        std::vector<LevelNode> next;
        for (size_t i = 0; i < level.size(); i++) {
            LevelNode& ln = level[i];
            Cand& c = chosen[i];
            if (!c.found) {
                float v = t.nodes[ln.node].leaf;
                for (size_t k = 0; k < ln.len; k++) preds[cur[ln.start + k]] += v;
                continue;
            }
            const uint16_t* col = C.bins.data() + (size_t)c.feat * C.n;
            size_t nl = partition_rows(cur.data() + ln.start, ln.len, nxt.data() + ln.start, col,
                                       C.cuts.missing(c.feat), c);
            leaf_count++;
            float lv, rv;
            Bounds lb, rb;
            child_values(c, q, p, ln.bounds, C.P.mono_of(c.feat), lv, rv, lb, rb);
            int l, r;
            t.split_leaf(ln.node, c.feat, c.is_cat ? 0.0f : C.cuts.threshold(c.feat, c.bin), c.missing_left, c.gain,
                         lv, q.hess_f32(c.left), rv, q.hess_f32(c.right), l, r);
            if (c.is_cat) {
                t.nodes[ln.node].is_cat = true;
                t.nodes[ln.node].cats = c.cats;
                t.nodes[ln.node].cond = std::numeric_limits<float>::denorm_min();
            }
            size_t nr = ln.len - nl;
            int small = nl <= nr ? 0 : 1;
            int slot = (int)next.size();
            LevelNode L{l, ln.start, nl, c.left, -1, -1, lb};
            LevelNode R{r, ln.start + nl, nr, c.right, -1, -1, rb};
            if (small == 0) { R.hist_from = (int)i; R.sibling = slot; }
            else { L.hist_from = (int)i; L.sibling = slot + 1; }
            next.push_back(L);
            next.push_back(R);
        }
        parent_hists = std::move(hists);
        std::swap(cur, nxt);
        level = std::move(next);
    }
    for (const LevelNode& ln : level) {
        float v = t.nodes[ln.node].leaf;
        for (size_t k = 0; k < ln.len; k++) preds[cur[ln.start + k]] += v;
    }
    return t;
}

// Row-sharded depthwise growth with threads as ranks: the device engine's
// multi-GPU design restated on the CPU, to show it grows the reference's
// trees.  Rank r holds rows [n r / N, n (r + 1) / N) and its own row buffers;
// per level every rank (a thread) builds partial histograms of the accumulate
// nodes over its own rows, a fake collective sums them modulo 2^64 in rank
// order, and each rank partitions its own rows.  No row counts are
// exchanged: the accumulated child is the one with the smaller global
// hessian sum (left on ties), which changes which histogram is built, never
// its integers.  With feature_sharded the sum is a reduce-scatter by feature
// range: rank r scores splits on its own features only, and the per-node
// winners are gathered in rank order, a strictly greater gain replacing the
// current winner, so equal gains keep the lower feature as best_split does.
struct ShardMode {
    int ranks = 0;
    bool feature_sharded = false;
};
thread_local ShardMode g_shard;

Tree build_tree_depthwise_sharded(Ctx& C, const std::vector<FX>& gpair, FX root_sum, const Quantizer& q,
                                  std::vector<float>& preds, const uint8_t* enabled, int N, bool feat_shard) {
    const rc_params& p = C.P.p;
    const uint32_t F = C.cuts.n_feats();
    Tree t;
    int root = t.push_leaf(leaf_of(root_sum, q, p), q.hess_f32(root_sum));
    std::vector<uint64_t> lo(N + 1);
    for (int r = 0; r <= N; r++) lo[r] = C.n * (uint64_t)r / (uint64_t)N;
    std::vector<std::vector<uint32_t>> cur(N), nxt(N);
    for (int r = 0; r < N; r++) {
        for (uint64_t i = lo[r]; i < lo[r + 1]; i++) cur[r].push_back((uint32_t)i);
        nxt[r].resize(cur[r].size());
    }
    struct SNode {
        int node;
        std::vector<size_t> start, len;  // per rank
        FX sum;
        int hist_from, sibling;
        Bounds bounds;
    };
    std::vector<SNode> level(1);
    level[0].node = root;
    level[0].sum = root_sum;
    level[0].hist_from = level[0].sibling = -1;
    level[0].bounds = kUnbounded;
    for (int r = 0; r < N; r++) {
        level[0].start.push_back(0);
        level[0].len.push_back(cur[r].size());
    }
    std::vector<std::vector<FX>> parent_hists;
    uint32_t leaf_count = 1;
    std::vector<uint32_t> feat_lo(N + 1);
    for (int r = 0; r <= N; r++) feat_lo[r] = (uint32_t)((uint64_t)F * r / N);
    for (uint32_t depth = 0; depth < p.max_depth; depth++) {
        if (level.empty() || (p.max_leaves != 0 && leaf_count >= p.max_leaves)) break;
        std::vector<size_t> acc;
        for (size_t i = 0; i < level.size(); i++)
            if (level[i].hist_from < 0) acc.push_back(i);
        // every rank: partial histograms of the accumulate nodes over its rows
        std::vector<std::vector<std::vector<FX>>> part(N);
        std::vector<std::thread> ranks;
        for (int r = 0; r < N; r++) {
            ranks.emplace_back([&, r] {
                part[r].assign(acc.size(), std::vector<FX>(C.total_bins, FX{0, 0}));
                std::vector<const uint32_t*> rows;
                std::vector<size_t> lens;
                std::vector<FX*> outs;
                for (size_t k = 0; k < acc.size(); k++) {
                    rows.push_back(cur[r].data() + level[acc[k]].start[r]);
                    lens.push_back(level[acc[k]].len[r]);
                    outs.push_back(part[r][k].data());
                }
                hist_nodes(C.bins, C.n, C.cuts, C.hoff, gpair, rows, lens, outs, 1);
            });
        }
        for (auto& th : ranks) th.join();
        // the collective: sums in rank order (all-reduce; a reduce-scatter
        // delivers the same sums for each rank's own feature range)
        std::vector<std::vector<FX>> hists(level.size());
        for (size_t k = 0; k < acc.size(); k++) {
            std::vector<FX>& h = hists[acc[k]];
            h = std::move(part[0][k]);
            for (int r = 1; r < N; r++)
                for (uint32_t b = 0; b < C.total_bins; b++) h[b] = fx_add(h[b], part[r][k][b]);
        }
        for (size_t i = 0; i < level.size(); i++) {
            if (level[i].hist_from >= 0) {
                std::vector<FX>& ph = parent_hists[level[i].hist_from];
                const std::vector<FX>& sib = hists[level[i].sibling];
                for (uint32_t b = 0; b < C.total_bins; b++) ph[b] = fx_sub(ph[b], sib[b]);
                hists[i] = std::move(ph);
            }
        }
        std::vector<Cand> chosen(level.size());
        for (size_t i = 0; i < level.size(); i++) {
            if (!feat_shard) {
                chosen[i] = best_split(hists[i].data(), F, C.hoff.data(), level[i].sum, q, C.P, level[i].bounds,
                                       enabled);
                continue;
            }
            Cand best;
            for (int r = 0; r < N; r++) {  // gather of the per-rank winners, in rank order
                std::vector<uint8_t> own(F, 0);
                for (uint32_t f = feat_lo[r]; f < feat_lo[r + 1]; f++) own[f] = enabled ? enabled[f] : 1;
                Cand c = best_split(hists[i].data(), F, C.hoff.data(), level[i].sum, q, C.P, level[i].bounds,
                                    own.data());
                if (c.found && (!best.found || c.gain > best.gain)) best = c;
            }
            chosen[i] = best;
        }
        if (p.max_leaves != 0) {
            uint32_t remaining = p.max_leaves > leaf_count ? p.max_leaves - leaf_count : 0;
            for (Cand& c : chosen) {
                if (!c.found) continue;
                if (remaining == 0) c.found = false; else remaining--;
            }
        }
        std::vector<SNode> next;
        for (size_t i = 0; i < level.size(); i++) {
            SNode& ln = level[i];
            Cand& c = chosen[i];
            if (!c.found) {
                float v = t.nodes[ln.node].leaf;
                for (int r = 0; r < N; r++)
                    for (size_t k = 0; k < ln.len[r]; k++) preds[cur[r][ln.start[r] + k]] += v;
                continue;
            }
            const uint16_t* col = C.bins.data() + (size_t)c.feat * C.n;
            SNode L, Rn;
            for (int r = 0; r < N; r++) {  // each rank partitions its own rows
                size_t nl = partition_rows(cur[r].data() + ln.start[r], ln.len[r], nxt[r].data() + ln.start[r], col,
                                           C.cuts.missing(c.feat), c);
                L.start.push_back(ln.start[r]);
                L.len.push_back(nl);
                Rn.start.push_back(ln.start[r] + nl);
                Rn.len.push_back(ln.len[r] - nl);
            }
            leaf_count++;
            float lv, rv;
            Bounds lb, rb;
            child_values(c, q, p, ln.bounds, C.P.mono_of(c.feat), lv, rv, lb, rb);
            int l, r;
            t.split_leaf(ln.node, c.feat, c.is_cat ? 0.0f : C.cuts.threshold(c.feat, c.bin), c.missing_left, c.gain,
                         lv, q.hess_f32(c.left), rv, q.hess_f32(c.right), l, r);
            if (c.is_cat) {
                t.nodes[ln.node].is_cat = true;
                t.nodes[ln.node].cats = c.cats;
                t.nodes[ln.node].cond = std::numeric_limits<float>::denorm_min();
            }
            // the smaller child by global hessian sum (signed compare, as the device does)
            const int small = c.left.h <= c.right.h ? 0 : 1;
            const int slot = (int)next.size();
            L.node = l; L.sum = c.left; L.bounds = lb; L.hist_from = L.sibling = -1;
            Rn.node = r; Rn.sum = c.right; Rn.bounds = rb; Rn.hist_from = Rn.sibling = -1;
            if (small == 0) { Rn.hist_from = (int)i; Rn.sibling = slot; }
            else { L.hist_from = (int)i; L.sibling = slot + 1; }
            next.push_back(std::move(L));
            next.push_back(std::move(Rn));
        }
        parent_hists = std::move(hists);
        std::swap(cur, nxt);
        level = std::move(next);
    }
    for (const SNode& ln : level) {
        float v = t.nodes[ln.node].leaf;
        for (int r = 0; r < N; r++)
            for (size_t k = 0; k < ln.len[r]; k++) preds[cur[r][ln.start[r] + k]] += v;
    }
    return t;
}

// training/lossguide.rs:506-700 grow (best-first).
Tree build_tree_lossguide(Ctx& C, const std::vector<FX>& gpair, FX root_sum, const Quantizer& q,
                          std::vector<float>& preds, const uint8_t* enabled) {
    const rc_params& p = C.P.p;
    Tree t;
    int root = t.push_leaf(leaf_of(root_sum, q, p), q.hess_f32(root_sum));
    std::vector<uint32_t> rows(C.n), buf;
    for (uint64_t i = 0; i < C.n; i++) rows[i] = (uint32_t)i;
    struct Leaf { int id; size_t start, len; uint32_t depth; FX sum; Bounds bounds; std::vector<FX> hist; };
    struct Pending { Leaf leaf; Cand split; };
    auto cmp = [](const Pending& a, const Pending& b) {  // lossguide.rs:46-53: gain, then lower id first
        // total_cmp on f32
        int32_t ia, ib;
        std::memcpy(&ia, &a.split.gain, 4);
        std::memcpy(&ib, &b.split.gain, 4);
        ia ^= (int32_t)(((uint32_t)(ia >> 31)) >> 1);
        ib ^= (int32_t)(((uint32_t)(ib >> 31)) >> 1);
        if (ia != ib) return ia < ib;
        return a.leaf.id > b.leaf.id;
    };
    std::vector<Pending> heap;
    auto finish = [&](const Leaf& l) {
        float v = t.nodes[l.id].leaf;
        for (size_t k = 0; k < l.len; k++) preds[rows[l.start + k]] += v;
    };
    // Evaluate leaves: histograms (the smaller child accumulates, the larger
    // subtracts it from its parent) and best splits (lossguide.rs:72-310).
    auto evaluate = [&](std::vector<Leaf> leaves, std::vector<FX>* parent_hist) {
        if (leaves.size() == 2 && parent_hist && !parent_hist->empty()) {
            int small = leaves[0].len > leaves[1].len ? 1 : 0;
            leaves[small].hist.assign(C.total_bins, FX{0, 0});
            std::vector<const uint32_t*> r{rows.data() + leaves[small].start};
            std::vector<size_t> ln{leaves[small].len};
            std::vector<FX*> o{leaves[small].hist.data()};
            hist_nodes(C.bins, C.n, C.cuts, C.hoff, gpair, r, ln, o, C.nth);
            std::vector<FX>& big = *parent_hist;
            for (uint32_t k = 0; k < C.total_bins; k++) big[k] = fx_sub(big[k], leaves[small].hist[k]);
            leaves[1 - small].hist = std::move(big);
        } else {
            std::vector<const uint32_t*> r;
            std::vector<size_t> ln;
            std::vector<FX*> o;
            for (Leaf& l : leaves) {
                l.hist.assign(C.total_bins, FX{0, 0});
                r.push_back(rows.data() + l.start);
                ln.push_back(l.len);
                o.push_back(l.hist.data());
            }
            hist_nodes(C.bins, C.n, C.cuts, C.hoff, gpair, r, ln, o, C.nth);
        }
        for (Leaf& l : leaves) {
            Cand c = best_split(l.hist.data(), C.cuts.n_feats(), C.hoff.data(), l.sum, q, C.P, l.bounds, enabled);
            if (c.found) {
                heap.push_back({std::move(l), c});
                std::push_heap(heap.begin(), heap.end(), cmp);
            } else {
                finish(l);
            }
        }
    };
    Leaf rl{root, 0, (size_t)C.n, 0, root_sum, kUnbounded, {}};
    if (p.max_depth == 0 || p.max_leaves == 1) finish(rl);
    else evaluate({std::move(rl)}, nullptr);
    uint32_t leaf_count = 1;
    while (p.max_leaves == 0 || leaf_count < p.max_leaves) {
        if (heap.empty()) break;
        std::pop_heap(heap.begin(), heap.end(), cmp);
        Pending pd = std::move(heap.back());
        heap.pop_back();
        Leaf& leaf = pd.leaf;
        Cand& c = pd.split;
        buf.resize(leaf.len);
        const uint16_t* col = C.bins.data() + (size_t)c.feat * C.n;
        size_t nl = partition_rows(rows.data() + leaf.start, leaf.len, buf.data(), col, C.cuts.missing(c.feat), c);
        std::copy(buf.begin(), buf.end(), rows.begin() + leaf.start);
        float lv, rv;
        Bounds lb, rb;
        child_values(c, q, p, leaf.bounds, C.P.mono_of(c.feat), lv, rv, lb, rb);
        int l, r;
        t.split_leaf(leaf.id, c.feat, c.is_cat ? 0.0f : C.cuts.threshold(c.feat, c.bin), c.missing_left, c.gain, lv,
                     q.hess_f32(c.left), rv, q.hess_f32(c.right), l, r);
        if (c.is_cat) {
            t.nodes[leaf.id].is_cat = true;
            t.nodes[leaf.id].cats = c.cats;
            t.nodes[leaf.id].cond = std::numeric_limits<float>::denorm_min();
        }
        leaf_count++;
        uint32_t depth = leaf.depth + 1;
        std::vector<Leaf> children;
        children.push_back({l, leaf.start, nl, depth, c.left, lb, {}});
        children.push_back({r, leaf.start + nl, leaf.len - nl, depth, c.right, rb, {}});
        if (depth == p.max_depth || leaf_count == p.max_leaves) {
            for (const Leaf& ch : children) finish(ch);
        } else {
            evaluate(std::move(children), &leaf.hist);
        }
    }
    for (const Pending& pd : heap) finish(pd.leaf);
    return t;
}

// training/mod.rs:2564-2800 train_multiclass_rounds (exact, host gradients):
// per round one softmax gradient of all K classes from the round's starting
// margins; then for class k = 0..K-1 the tree with index round*K + k keys the
// row sampling and colsample_bytree, its gradient column is masked, bounded
// and quantized, and the tree (the single-output builder) updates the class's
// margins before the next class's tree.
void train_multiclass(Ctx& C, Model* m, const float* y, const float* w, uint64_t n, uint32_t F) {
    const rc_params& p = C.P.p;
    const uint32_t K = p.num_class;
    m->class_margins = std::isnan(p.base_score) ? initial_class_margins(y, n, w, K)
                                                : std::vector<float>(K, p.base_score);
    m->base_score = m->class_margins[0];
    std::vector<std::vector<float>> preds(K);
    for (uint32_t k = 0; k < K; k++) preds[k].assign(n, m->class_margins[k]);
    std::vector<GP> gp((size_t)K * n);
    std::vector<GP> col(n);
    std::vector<FX> fixed(n);
    const uint64_t sub_th = threshold_for(p.subsample);
    const int nth = C.nth;
    for (uint32_t round = 0; round < p.n_rounds; round++) {
        auto t_round = std::chrono::steady_clock::now();
#pragma omp parallel num_threads(nth)
        {
            std::vector<float> mr(K);
            std::vector<GP> out(K);
#pragma omp for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) {
                for (uint32_t k = 0; k < K; k++) mr[k] = preds[k][i];
                softmax_row(mr.data(), K, y[i], w ? w[i] : 1.0f, out.data());
                for (uint32_t k = 0; k < K; k++) gp[(size_t)k * n + i] = out[k];
            }
        }
        for (uint32_t k = 0; k < K; k++) {
            const uint64_t tree = (uint64_t)round * K + k;
            double mg = 0.0, mh = 0.0;
#pragma omp parallel for reduction(max : mg, mh) num_threads(nth)
            for (int64_t i = 0; i < (int64_t)n; i++) {  // mod.rs:4811-4842 mask_and_bounds
                GP g = gp[(size_t)k * n + i];
                if (sub_th != UINT64_MAX && (row_hash((uint64_t)i, p.seed, tree) >> 11) >= sub_th) g = {0.0f, 0.0f};
                col[i] = g;
                mg = std::max(mg, finite_abs(g.g));
                mh = std::max(mh, finite_abs(g.h));
            }
            if (!std::isfinite(mg) || !std::isfinite(mh)) throw std::runtime_error("non-finite gradient or Hessian");
            Quantizer q = Quantizer::from_scales(pow2_scale(mg, n), pow2_scale(mh, n));
            int64_t sg = 0, sh = 0;
#pragma omp parallel for reduction(+ : sg, sh) num_threads(nth)
            for (int64_t i = 0; i < (int64_t)n; i++) {
                FX f = q.to_fixed(col[i]);
                fixed[i] = f;
                sg = (int64_t)((uint64_t)sg + (uint64_t)f.g);
                sh = (int64_t)((uint64_t)sh + (uint64_t)f.h);
            }
            std::vector<uint8_t> enabled;
            if (p.colsample_bytree < 1.0f) {
                enabled.assign(F, 0);
                for (uint32_t f : sample_features(F, p.colsample_bytree, p.seed, tree)) enabled[f] = 1;
            }
            const uint8_t* en = enabled.empty() ? nullptr : enabled.data();
            Tree t = p.grow_policy == 1 ? build_tree_lossguide(C, fixed, FX{sg, sh}, q, preds[k], en)
                                        : build_tree_depthwise(C, fixed, FX{sg, sh}, q, preds[k], en);
            m->trees.push_back(std::move(t));
        }
        g_round_s.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t_round).count());
    }
}

Model* train_impl(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const rc_params* rp) {
    Params P;
    P.p = *rp;
    if (rp->monotone) P.mono.assign(rp->monotone, rp->monotone + F);
    if (rp->categorical) {
        bool any = false;
        for (uint32_t f = 0; f < F; f++) any |= rp->categorical[f] != 0;
        if (any) P.cat.assign(rp->categorical, rp->categorical + F);
    }
    const rc_params& p = P.p;
    auto t_setup = std::chrono::steady_clock::now();
    g_round_s.clear();
    if (n == 0 || F == 0) { g_err = "training data must have at least one row and one feature"; return nullptr; }
    if (p.max_depth > 14) { g_err = "max_depth must be in 0..=14"; return nullptr; }
    int nth = n_threads(p.nthread);
    Cuts cuts = sketch_cuts(X, n, F, p.max_bin, w, P.cat.empty() ? nullptr : P.cat.data(), nth);
    std::vector<uint16_t> bins;
    quantize_cols(X, n, F, cuts, bins, nth);
    Ctx C{P, cuts, bins, n, {}, 0, nth};
    C.hoff.push_back(0);
    for (uint32_t f = 0; f < F; f++) C.hoff.push_back(C.hoff.back() + cuts.n_bins(f));
    C.total_bins = C.hoff.back();

    Model* m = new Model();
    m->n_features = F;
    m->objective = p.objective;
    m->scale_pos_weight = p.scale_pos_weight;
    if (!P.cat.empty()) m->feature_types = P.cat;
    // gradient weights: sample weight x scale_pos_weight on positives (mod.rs:5470-5495)
    std::vector<float> gw;
    const float* gwp = w;
    if (p.scale_pos_weight != 1.0f) {
        gw.resize(n);
        for (uint64_t i = 0; i < n; i++) {
            float wi = w ? w[i] : 1.0f;
            gw[i] = y[i] == 1.0f ? wi * p.scale_pos_weight : wi;
        }
        gwp = gw.data();
    }
    if (p.objective >= 2) {  // objective.rs:642-690 validate_labels
        if (p.num_class < 2) { g_err = "multi:softprob / multi:softmax need num_class >= 2"; delete m; return nullptr; }
        for (uint64_t i = 0; i < n; i++)
            if (!(y[i] >= 0.0f && y[i] < (float)p.num_class && y[i] == std::trunc(y[i]))) {
                g_err = "multiclass labels must be integers in [0, num_class)";
                delete m;
                return nullptr;
            }
        g_setup_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_setup).count();
        train_multiclass(C, m, y, w, n, F);
        return m;
    }
    m->base_score = std::isnan(p.base_score)
                        ? initial_base_score(p.objective, y, n, w, p.scale_pos_weight != 1.0f ? gwp : w,
                                             p.scale_pos_weight)
                        : p.base_score;
    float margin = base_margin(p.objective, m->base_score);
    std::vector<float> preds(n, margin);
    std::vector<GP> gp(n);
    std::vector<FX> fixed(n);
    uint64_t sub_th = threshold_for(p.subsample);
    g_setup_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_setup).count();
    for (uint32_t round = 0; round < p.n_rounds; round++) {
        auto t_round = std::chrono::steady_clock::now();
        // gradient (mod.rs:5624-5634) + row sampling mask + bounds (mod.rs:4811-4842)
        double mg = 0.0, mh = 0.0;
#pragma omp parallel for reduction(max : mg, mh) num_threads(nth)
        for (int64_t i = 0; i < (int64_t)n; i++) {
            GP g = gradient_of(preds[i], y[i], p.objective);
            if (gwp) { g.g = g.g * gwp[i]; g.h = g.h * gwp[i]; }
            if (sub_th != UINT64_MAX && (row_hash((uint64_t)i, p.seed, round) >> 11) >= sub_th) g = {0.0f, 0.0f};
            gp[i] = g;
            mg = std::max(mg, finite_abs(g.g));
            mh = std::max(mh, finite_abs(g.h));
        }
        if (!std::isfinite(mg) || !std::isfinite(mh)) { g_err = "non-finite gradient or Hessian"; delete m; return nullptr; }
        Quantizer q = Quantizer::from_scales(pow2_scale(mg, n), pow2_scale(mh, n));
        int64_t sg = 0, sh = 0;
#pragma omp parallel for reduction(+ : sg, sh) num_threads(nth)
        for (int64_t i = 0; i < (int64_t)n; i++) {
            FX f = q.to_fixed(gp[i]);
            fixed[i] = f;
            sg = (int64_t)((uint64_t)sg + (uint64_t)f.g);
            sh = (int64_t)((uint64_t)sh + (uint64_t)f.h);
        }
        FX root_sum{sg, sh};
        std::vector<uint8_t> enabled;
        if (p.colsample_bytree < 1.0f) {
            enabled.assign(F, 0);
            for (uint32_t f : sample_features(F, p.colsample_bytree, p.seed, round)) enabled[f] = 1;
        }
        const uint8_t* en = enabled.empty() ? nullptr : enabled.data();
        Tree t = p.grow_policy == 1 ? build_tree_lossguide(C, fixed, root_sum, q, preds, en)
                 : g_shard.ranks > 1
                     ? build_tree_depthwise_sharded(C, fixed, root_sum, q, preds, en, g_shard.ranks,
                                                    g_shard.feature_sharded)
                     : build_tree_depthwise(C, fixed, root_sum, q, preds, en);
        m->trees.push_back(std::move(t));
        g_round_s.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t_round).count());
    }
    return m;
}

// ---------------------------------------------------------------- JSON
// model/tree.rs:600-750 + 1167-1257 (serde field order); float text follows
// serde_json's shortest round-trip f32 form, base_score Rust's Display.
void shortest_digits(float v, std::string& digits, int& exp10) {
    // digits d1d2..dk and exponent so that v = 0.d1..dk * 10^exp10
    char buf[64];
    auto r = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::scientific);
    std::string s(buf, r.ptr);
    size_t e = s.find('e');
    std::string mant = s.substr(0, e);
    int ex = std::atoi(s.c_str() + e + 1);
    digits.clear();
    for (char ch : mant) if (ch >= '0' && ch <= '9') digits.push_back(ch);
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    exp10 = ex + 1;
}

std::string fmt_f32_json(float v) {  // serde_json / ryu layout of an f32
    if (!std::isfinite(v)) return "null";
    std::string out;
    if (std::signbit(v)) { out.push_back('-'); v = -v; }
    if (v == 0.0f) return out + "0.0";
    std::string d;
    int kk;
    shortest_digits(v, d, kk);
    int len = (int)d.size();
    int k = kk - len;
    if (0 <= k && kk <= 13) {
        out += d;
        out.append((size_t)(kk - len), '0');
        out += ".0";
    } else if (0 < kk && kk <= 13) {
        out += d.substr(0, (size_t)kk);
        out.push_back('.');
        out += d.substr((size_t)kk);
    } else if (-6 < kk && kk <= 0) {
        out += "0.";
        out.append((size_t)(-kk), '0');
        out += d;
    } else if (len == 1) {
        out += d;
        out.push_back('e');
        out += std::to_string(kk - 1);
    } else {
        out += d.substr(0, 1);
        out.push_back('.');
        out += d.substr(1);
        out.push_back('e');
        out += std::to_string(kk - 1);
    }
    return out;
}

std::string fmt_f32_display(float v) {  // Rust `impl Display for f32`
    if (std::isnan(v)) return "NaN";
    std::string out;
    if (std::signbit(v)) { out.push_back('-'); v = -v; }
    if (std::isinf(v)) return out + "inf";
    if (v == 0.0f) return out + "0";
    std::string d;
    int kk;
    shortest_digits(v, d, kk);
    int len = (int)d.size();
    if (kk <= 0) {
        out += "0.";
        out.append((size_t)(-kk), '0');
        out += d;
    } else if (kk >= len) {
        out += d;
        out.append((size_t)(kk - len), '0');
    } else {
        out += d.substr(0, (size_t)kk);
        out.push_back('.');
        out += d.substr((size_t)kk);
    }
    return out;
}

template <class T, class F> void json_array(std::string& o, const std::vector<T>& v, F f) {
    o.push_back('[');
    for (size_t i = 0; i < v.size(); i++) { if (i) o.push_back(','); o += f(v[i]); }
    o.push_back(']');
}

std::string model_json(const Model& m) {
    std::string o;
    o.reserve(1 << 16);
    o += "{\"version\":[2,0,0],\"learner\":{\"attributes\":{},\"feature_names\":[],\"feature_types\":";
    bool any_cat = false;
    for (uint8_t c : m.feature_types) any_cat |= c != 0;
    if (any_cat) {
        std::vector<std::string> ft;
        for (uint32_t f = 0; f < m.n_features; f++)
            ft.push_back(f < m.feature_types.size() && m.feature_types[f] ? "\"c\"" : "\"q\"");
        json_array(o, ft, [](const std::string& s) { return s; });
    } else {
        o += "[]";
    }
    size_t nt = m.trees.size();
    const size_t K = m.class_margins.empty() ? 1 : m.class_margins.size();
    o += ",\"gradient_booster\":{\"name\":\"gbtree\",\"model\":{\"gbtree_model_param\":{\"num_trees\":\"" +
         std::to_string(nt) + "\",\"num_parallel_tree\":\"1\"},\"iteration_indptr\":[";
    for (size_t i = 0; i < nt; i += K) { if (i) o.push_back(','); o += std::to_string(i); }  // tree.rs:690-697
    if (nt) o.push_back(',');
    o += std::to_string(nt);
    o += "],\"tree_info\":[";
    for (size_t i = 0; i < nt; i++) { if (i) o.push_back(','); o += std::to_string(i % K); }
    o += "],\"trees\":[";
    auto fj = [](float v) { return fmt_f32_json(v); };
    auto ij = [](int64_t v) { return std::to_string(v); };
    for (size_t ti = 0; ti < nt; ti++) {
        const Tree& t = m.trees[ti];
        size_t nn = t.nodes.size();
        std::vector<float> bw, lc, sc, sh;
        std::vector<int64_t> dl, lch, rch, par(nn, 2147483647), si, st(nn, 0), cats, cnodes, cseg, csz;
        for (size_t i = 0; i < nn; i++) {
            const Node& nd = t.nodes[i];
            lch.push_back(nd.left);
            rch.push_back(nd.right);
            dl.push_back(nd.default_left ? 1 : 0);
            lc.push_back(nd.gain);
            sh.push_back(nd.hess);
            if (nd.is_leaf) {
                sc.push_back(nd.leaf);
                si.push_back(0);
                bw.push_back(nd.leaf);
            } else {
                sc.push_back(nd.cond);
                si.push_back(nd.feat);
                bw.push_back(0.0f);
                par[nd.left] = (int64_t)i;
                par[nd.right] = (int64_t)i;
                if (nd.is_cat) {
                    st[i] = 1;
                    cnodes.push_back((int64_t)i);
                    cseg.push_back((int64_t)cats.size());
                    int64_t cnt = 0;
                    for (size_t wi = 0; wi < nd.cats.size(); wi++)
                        for (int b = 0; b < 32; b++)
                            if ((nd.cats[wi] >> b) & 1u) { cats.push_back((int64_t)(wi * 32 + b)); cnt++; }
                    csz.push_back(cnt);
                }
            }
        }
        if (ti) o.push_back(',');
        o += "{\"base_weights\":"; json_array(o, bw, fj);
        o += ",\"categories\":"; json_array(o, cats, ij);
        o += ",\"categories_nodes\":"; json_array(o, cnodes, ij);
        o += ",\"categories_segments\":"; json_array(o, cseg, ij);
        o += ",\"categories_sizes\":"; json_array(o, csz, ij);
        o += ",\"default_left\":"; json_array(o, dl, ij);
        o += ",\"id\":" + std::to_string(ti);
        o += ",\"left_children\":"; json_array(o, lch, ij);
        o += ",\"loss_changes\":"; json_array(o, lc, fj);
        o += ",\"parents\":"; json_array(o, par, ij);
        o += ",\"right_children\":"; json_array(o, rch, ij);
        o += ",\"split_conditions\":"; json_array(o, sc, fj);
        o += ",\"split_indices\":"; json_array(o, si, ij);
        o += ",\"split_type\":"; json_array(o, st, ij);
        o += ",\"sum_hessian\":"; json_array(o, sh, fj);
        o += ",\"tree_param\":{\"num_deleted\":\"0\",\"num_feature\":\"" + std::to_string(m.n_features) +
             "\",\"num_nodes\":\"" + std::to_string(nn) + "\",\"size_leaf_vector\":\"1\"}}";
    }
    std::string base = fmt_f32_display(m.base_score);
    if (!m.class_margins.empty()) {  // tree.rs:704-720: the vector form "[a,b,c]"
        base = "[";
        for (size_t k = 0; k < K; k++) { if (k) base.push_back(','); base += fmt_f32_display(m.class_margins[k]); }
        base.push_back(']');
    }
    o += "]}},\"learner_model_param\":{\"base_score\":\"" + base +
         "\",\"boost_from_average\":\"1\",\"num_class\":\"" + std::to_string(m.class_margins.empty() ? 0 : K) +
         "\",\"num_feature\":\"" + std::to_string(m.n_features) + "\",\"num_target\":\"1\"},\"objective\":{\"name\":\"";
    if (m.objective >= 2) {  // objective.rs:816-820 softmax_multiclass_param
        o += m.objective == 2 ? "multi:softprob" : "multi:softmax";
        o += "\",\"softmax_multiclass_param\":{\"num_class\":\"" + std::to_string(K) + "\"}}}}";
    } else {
        o += m.objective == 1 ? "binary:logistic" : "reg:squarederror";
        o += "\",\"reg_loss_param\":{\"scale_pos_weight\":\"" + fmt_f32_display(m.scale_pos_weight) + "\"}}}}";
    }
    return o;
}

// ---------------------------------------------------------------- TreeSHAP
// model/explain.rs:32-401, 478-728: 8-point QuadratureTreeSHAP.
constexpr int kPts = 8;
struct Rule { float nodes[kPts], weights[kPts]; };
double legendre(int n, double x) {  // explain.rs:121-134
    if (n == 0) return 1.0;
    double p0 = 1.0, p1 = x;
    for (int k = 2; k <= n; k++) {
        double kf = (double)k;
        double pk = ((2.0 * kf - 1.0) * x * p1 - (kf - 1.0) * p0) / kf;
        p0 = p1;
        p1 = pk;
    }
    return p1;
}
Rule make_rule() {  // explain.rs:141-169 MakeEndpointQuadrature
    Rule r{};
    const int n = kPts;
    const double pi = 3.14159265358979323846;
    for (int i = 0; i < n; i++) {
        double theta = pi * ((double)i + 0.75) / ((double)n + 0.5);
        double x = std::cos(theta);
        for (int it = 0; it < 64; it++) {
            double pn = legendre(n, x);
            double dpn = (double)n * (x * pn - legendre(n - 1, x)) / (x * x - 1.0);
            double dx = pn / dpn;
            x -= dx;
            if (std::fabs(dx) < 1e-15) break;
        }
        double pn = legendre(n, x);
        double dpn = (double)n * (x * pn - legendre(n - 1, x)) / (x * x - 1.0);
        double wq = 2.0 / ((1.0 - x * x) * dpn * dpn);
        double s = 0.5 * (x + 1.0);
        double ws = 0.5 * wq;
        int out = n - 1 - i;
        r.nodes[out] = (float)(s * s);
        r.weights[out] = (float)(2.0 * s * ws);
    }
    return r;
}
const Rule& rule() { static Rule r = make_rule(); return r; }

inline float branch_weight(float cover, float parent) {  // explain.rs:182-192
    if (parent <= 0.0f) return 0.5f;
    float w = cover / parent;
    return w < 1e-12f ? 1e-12f : w;
}
inline float extract_delta(const Rule& R, const float* h, float pe, float px) {  // explain.rs:198-216
    float acc = 0.0f;
    if (pe != 1.0f) {
        float a = pe - 1.0f;
        for (int i = 0; i < kPts; i++) acc += a * h[i] / (1.0f + a * R.nodes[i]);
    }
    if (px != 1.0f) {
        float a = px - 1.0f;
        for (int i = 0; i < kPts; i++) acc -= a * h[i] / (1.0f + a * R.nodes[i]);
    }
    return acc;
}
constexpr float kUnseen = -999.0f;
struct ShapRunner {  // explain.rs:302-400 Runner with the additive formulation
    const std::vector<Node>& nodes;
    const float* x;
    const Rule& R;
    float* path_prob;
    float* phi;
    void visit_child(int split, int child, float cw, bool sat, const float* c, float wp, float* out_h) {
        uint32_t feat = nodes[split].feat;
        float p_old = path_prob[feat];
        float pe = sat ? (p_old == kUnseen ? 1.0f / cw : p_old / cw) : 0.0f;
        float cc[kPts];
        float ae = pe - 1.0f;
        for (int i = 0; i < kPts; i++) cc[i] = c[i] * (1.0f + ae * R.nodes[i]);
        if (p_old != kUnseen) {
            float ao = p_old - 1.0f;
            if (ao != 0.0f)
                for (int i = 0; i < kPts; i++) cc[i] /= 1.0f + ao * R.nodes[i];
        }
        path_prob[feat] = pe;
        run_node(child, cc, wp * cw, out_h);
        float px = p_old == kUnseen ? 1.0f : p_old;
        phi[feat] += extract_delta(R, out_h, pe, px);
        path_prob[feat] = p_old;
    }
    void run_node(int idx, const float* c, float wp, float* out_h) {
        const Node& nd = nodes[idx];
        if (nd.is_leaf) {
            float ls = wp * nd.leaf;
            for (int i = 0; i < kPts; i++) out_h[i] = c[i] * ls * R.weights[i];
            return;
        }
        float lw = branch_weight(nodes[nd.left].hess, nd.hess);
        float rw = branch_weight(nodes[nd.right].hess, nd.hess);
        bool gl = node_goes_left(nd, x[nd.feat]);
        float rh[kPts] = {0};
        visit_child(idx, nd.left, lw, gl, c, wp, out_h);
        visit_child(idx, nd.right, rw, !gl, c, wp, rh);
        for (int i = 0; i < kPts; i++) out_h[i] += rh[i];
    }
};

// explain.rs:218-246 extract_interaction_delta
inline float extract_interaction_delta(const Rule& R, const float* h, float pe, float px, float q) {
    if (q == 1.0f) return 0.0f;
    const float ap = q - 1.0f, ae = pe - 1.0f;
    float acc = 0.0f;
    if (px == 1.0f) {
        for (int i = 0; i < kPts; i++) {
            float edge = ae / (1.0f + ae * R.nodes[i]);
            acc += ap * h[i] * edge / (1.0f + ap * R.nodes[i]);
        }
    } else {
        const float ax = px - 1.0f;
        for (int i = 0; i < kPts; i++) {
            float edge = ae / (1.0f + ae * R.nodes[i]) - ax / (1.0f + ax * R.nodes[i]);
            acc += ap * h[i] * edge / (1.0f + ap * R.nodes[i]);
        }
    }
    return acc;
}

// explain.rs:267-301 Interaction formulation over the Runner of explain.rs:302-400
struct InteractionRunner {
    const std::vector<Node>& nodes;
    const float* x;
    const Rule& R;
    float* path_prob;
    std::vector<std::pair<uint32_t, float>>& path;
    float* diag;
    float* matrix;
    uint32_t ncols;
    void on_return(uint32_t feat, const float* h, float pe, float px) {
        diag[feat] += extract_delta(R, h, pe, px);
        // partners: the newest occurrence of every other feature on the live
        // path, newest to oldest; the current split (the newest entry) is skipped
        const size_t len = path.size();
        bool skipped_current = false;
        for (size_t i = len; i-- > 0;) {
            const uint32_t split = path[i].first;
            const float p_child = path[i].second;
            bool shadowed = false;
            for (size_t j = i + 1; j < len; j++)
                if (path[j].first == split) { shadowed = true; break; }
            if (shadowed) continue;
            if (!skipped_current && split == feat) { skipped_current = true; continue; }
            matrix[(size_t)feat * ncols + split] += extract_interaction_delta(R, h, pe, px, p_child);
        }
    }
    void visit_child(int split, int child, float cw, bool sat, const float* c, float wp, float* out_h) {
        uint32_t feat = nodes[split].feat;
        float p_old = path_prob[feat];
        float pe = sat ? (p_old == kUnseen ? 1.0f / cw : p_old / cw) : 0.0f;
        float cc[kPts];
        float ae = pe - 1.0f;
        for (int i = 0; i < kPts; i++) cc[i] = c[i] * (1.0f + ae * R.nodes[i]);
        if (p_old != kUnseen) {
            float ao = p_old - 1.0f;
            if (ao != 0.0f)
                for (int i = 0; i < kPts; i++) cc[i] /= 1.0f + ao * R.nodes[i];
        }
        path_prob[feat] = pe;
        path.push_back({feat, pe});
        run_node(child, cc, wp * cw, out_h);
        float px = p_old == kUnseen ? 1.0f : p_old;
        on_return(feat, out_h, pe, px);
        path.pop_back();
        path_prob[feat] = p_old;
    }
    void run_node(int idx, const float* c, float wp, float* out_h) {
        const Node& nd = nodes[idx];
        if (nd.is_leaf) {
            float ls = wp * nd.leaf;
            for (int i = 0; i < kPts; i++) out_h[i] = c[i] * ls * R.weights[i];
            return;
        }
        float lw = branch_weight(nodes[nd.left].hess, nd.hess);
        float rw = branch_weight(nodes[nd.right].hess, nd.hess);
        bool gl = node_goes_left(nd, x[nd.feat]);
        float rh[kPts] = {0};
        visit_child(idx, nd.left, lw, gl, c, wp, out_h);
        visit_child(idx, nd.right, rw, !gl, c, wp, rh);
        for (int i = 0; i < kPts; i++) out_h[i] += rh[i];
    }
};

// explain.rs:409-421 fill_node_means (float32, FillNodeMeanValues)
float fill_node_means(const std::vector<Node>& nodes, int idx, std::vector<float>& means) {
    const Node& nd = nodes[idx];
    float value;
    if (nd.is_leaf) {
        value = nd.leaf;
    } else {
        float result = fill_node_means(nodes, nd.left, means) * nodes[nd.left].hess;
        result += fill_node_means(nodes, nd.right, means) * nodes[nd.right].hess;
        value = result / nd.hess;
    }
    means[idx] = value;
    return value;
}

double root_mean(const std::vector<Node>& nodes, int idx) {  // explain.rs:412-426
    const Node& nd = nodes[idx];
    if (nd.is_leaf) return (double)nd.leaf;
    double lm = root_mean(nodes, nd.left), rm = root_mean(nodes, nd.right);
    if (nd.hess == 0.0f) return 0.5 * (lm + rm);
    return (lm * (double)nodes[nd.left].hess + rm * (double)nodes[nd.right].hess) / (double)nd.hess;
}

}  // namespace

// ==================================================================== C API
extern "C" {

void rc_default_params(rc_params* p) {  // types.rs:641-686 Default for TrainParams
    std::memset(p, 0, sizeof(*p));
    p->objective = 1;
    p->grow_policy = 0;
    p->n_rounds = 100;
    p->max_depth = 6;
    p->max_leaves = 0;
    p->max_bin = 255;
    p->eta = 0.3f;
    p->lambda = 1.0f;
    p->min_child_weight = 1.0f;
    p->scale_pos_weight = 1.0f;
    p->subsample = 1.0f;
    p->colsample_bytree = 1.0f;
    p->base_score = std::numeric_limits<float>::quiet_NaN();
    p->max_cat_to_onehot = 4;
    p->max_cat_threshold = 64;
}

const char* rc_last_error(void) { return g_err.c_str(); }

int32_t rc_last_timing(double* setup_s, double* round_s, int32_t cap) {
    if (setup_s) *setup_s = g_setup_s;
    const int32_t n = (int32_t)g_round_s.size();
    for (int32_t i = 0; i < n && i < cap; i++) round_s[i] = g_round_s[i];
    return n;
}

void* rc_train(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const rc_params* p) {
    try {
        return train_impl(X, n, F, y, w, p);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void* rc_train_sharded(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const rc_params* p,
                       int32_t n_ranks, int32_t feature_sharded) {
    if (n_ranks < 1 || (uint64_t)n_ranks > n) { g_err = "n_ranks must be in 1..=n"; return nullptr; }
    g_shard.ranks = n_ranks;
    g_shard.feature_sharded = feature_sharded != 0;
    void* m = rc_train(X, n, F, y, w, p);
    g_shard = ShardMode{};
    return m;
}

void rc_model_free(void* m) { delete (Model*)m; }
uint32_t rc_model_num_trees(void* m) { return (uint32_t)((Model*)m)->trees.size(); }
void rc_softmax_gradients(const float* margins, const float* y, const float* w, uint64_t n, uint32_t K, float* out) {
    std::vector<float> mr(K);
    std::vector<GP> g(K);
    for (uint64_t i = 0; i < n; i++) {
        for (uint32_t k = 0; k < K; k++) mr[k] = margins[(size_t)k * n + i];
        softmax_row(mr.data(), K, y[i], w ? w[i] : 1.0f, g.data());
        for (uint32_t k = 0; k < K; k++) {
            out[2 * ((size_t)k * n + i)] = g[k].g;
            out[2 * ((size_t)k * n + i) + 1] = g[k].h;
        }
    }
}

void rc_class_margins(const float* y, const float* w, uint64_t n, uint32_t K, float* out) {
    std::vector<float> v = initial_class_margins(y, n, w, K);
    for (uint32_t k = 0; k < K; k++) out[k] = v[k];
}

uint32_t rc_model_num_outputs(void* m) {
    const Model* M = (Model*)m;
    return M->class_margins.empty() ? 1u : (uint32_t)M->class_margins.size();
}
float rc_model_base_margin(void* m) { Model* M = (Model*)m; return base_margin(M->objective, M->base_score); }

void* rc_model_load(uint32_t n_trees, const uint32_t* tree_off, const int32_t* left, const int32_t* right,
                    const uint32_t* feat, const float* value, const uint8_t* default_left, const float* gain,
                    const float* hess, const uint64_t* cat_off, const uint32_t* cat_len, const uint32_t* cats,
                    uint32_t n_features, int32_t objective, float base_score, const float* class_margins,
                    uint32_t num_class, float scale_pos_weight, const uint8_t* feature_types) {
    try {
        auto m = std::make_unique<Model>();
        m->objective = objective;
        m->base_score = base_score;
        m->n_features = n_features;
        m->scale_pos_weight = scale_pos_weight;
        if (class_margins && num_class >= 2) m->class_margins.assign(class_margins, class_margins + num_class);
        if (feature_types) m->feature_types.assign(feature_types, feature_types + n_features);
        for (uint32_t t = 0; t < n_trees; t++) {
            const uint32_t b = tree_off[t], e = tree_off[t + 1];
            if (e <= b) throw std::runtime_error("a tree has no nodes");
            Tree T;
            T.nodes.resize(e - b);
            for (uint32_t i = b; i < e; i++) {
                Node& nd = T.nodes[i - b];
                nd.left = left[i];
                nd.right = right[i];
                nd.is_leaf = left[i] < 0;
                nd.default_left = default_left[i] != 0;
                nd.gain = gain[i];
                nd.hess = hess[i];
                if (nd.is_leaf) {
                    nd.leaf = value[i];
                    continue;
                }
                if (left[i] >= (int32_t)(e - b) || right[i] < 0 || right[i] >= (int32_t)(e - b))
                    throw std::runtime_error("child index out of range");
                if (feat[i] >= n_features) throw std::runtime_error("split feature out of range");
                nd.feat = feat[i];
                nd.cond = value[i];
                if (cat_len && cat_len[i]) {  // categorical.rs bitset: right-going codes
                    nd.is_cat = true;
                    for (uint32_t k = 0; k < cat_len[i]; k++) {
                        const uint32_t c = cats[cat_off[i] + k];
                        if (nd.cats.size() <= c / 32) nd.cats.resize(c / 32 + 1, 0u);
                        nd.cats[c / 32] |= 1u << (c % 32);
                    }
                }
            }
            m->trees.push_back(std::move(T));
        }
        return m.release();
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return nullptr;
    }
}

int64_t rc_model_json(void* m, char* buf, int64_t cap) {
    std::string s = model_json(*(Model*)m);
    if (buf && cap > 0) std::memcpy(buf, s.data(), (size_t)std::min<int64_t>(cap, (int64_t)s.size()));
    return (int64_t)s.size();
}

int64_t rc_model_tree(void* m, uint32_t t, uint32_t* feat, float* cond, int32_t* left, int32_t* right,
                      uint8_t* dl, float* leaf, uint8_t* is_leaf, float* gain, float* hess) {
    const Tree& T = ((Model*)m)->trees[t];
    for (size_t i = 0; i < T.nodes.size(); i++) {
        const Node& n = T.nodes[i];
        if (feat) feat[i] = n.feat;
        if (cond) cond[i] = n.cond;
        if (left) left[i] = n.left;
        if (right) right[i] = n.right;
        if (dl) dl[i] = n.default_left;
        if (leaf) leaf[i] = n.leaf;
        if (is_leaf) is_leaf[i] = n.is_leaf;
        if (gain) gain[i] = n.gain;
        if (hess) hess[i] = n.hess;
    }
    return (int64_t)T.nodes.size();
}

void rc_predict_margin(void* mp, const float* X, uint64_t n, float* out, int32_t nthread) {
    const Model& m = *(Model*)mp;
    float bm = base_margin(m.objective, m.base_score);
    int nth = n_threads(nthread);
    if (!m.class_margins.empty()) {  // tree.rs:468-480 predict_margins_upto: n x K, row-major
        const size_t K = m.class_margins.size();
#pragma omp parallel for schedule(static) num_threads(nth)
        for (int64_t r = 0; r < (int64_t)n; r++) {
            const float* x = X + (size_t)r * m.n_features;
            float* o = out + (size_t)r * K;
            for (size_t k = 0; k < K; k++) o[k] = m.class_margins[k];
            for (size_t t = 0; t < m.trees.size(); t++) o[t % K] += tree_leaf_value(m.trees[t], x);
        }
        return;
    }
#pragma omp parallel for schedule(static) num_threads(nth)
    for (int64_t r = 0; r < (int64_t)n; r++) {  // tree.rs:498-510 predict_margin_upto
        const float* x = X + (size_t)r * m.n_features;
        float acc = bm;
        for (const Tree& t : m.trees) acc += tree_leaf_value(t, x);
        out[r] = acc;
    }
}

void rc_shap(void* mp, const float* X, uint64_t n, float* out, int32_t nthread) {
    const Model& m = *(Model*)mp;
    const uint32_t F = m.n_features;
    const uint32_t nc = F + 1;
    const size_t K = m.class_margins.empty() ? 1 : m.class_margins.size();
    std::vector<double> sums(K, 0.0);  // explain.rs:527-539 group_root_mean, one group per output
    for (size_t t = 0; t < m.trees.size(); t++) sums[t % K] += root_mean(m.trees[t].nodes, 0);
    std::vector<float> group_mean(K), bias(K);
    for (size_t g = 0; g < K; g++) {
        group_mean[g] = (float)sums[g];
        bias[g] = m.class_margins.empty() ? base_margin(m.objective, m.base_score) : m.class_margins[g];
    }
    const Rule& R = rule();
    int nth = n_threads(nthread);
#pragma omp parallel num_threads(nth)
    {
        std::vector<float> path(F, kUnseen), tc(nc, 0.0f);
#pragma omp for schedule(dynamic, 16)
        for (int64_t r = 0; r < (int64_t)n; r++) {  // explain.rs:704-728 shap_row: groups g, trees g, g + K, ...
            const float* x = X + (size_t)r * F;
            for (size_t g = 0; g < K; g++) {
                float* p = out + ((size_t)r * K + g) * nc;
                for (uint32_t c = 0; c < nc; c++) p[c] = 0.0f;
                for (size_t ti = g; ti < m.trees.size(); ti += K) {
                    const Tree& t = m.trees[ti];
                    std::fill(tc.begin(), tc.end(), 0.0f);
                    if (!t.nodes[0].is_leaf) {
                        ShapRunner run{t.nodes, x, R, path.data(), tc.data()};
                        float ones[kPts], h[kPts];
                        for (int i = 0; i < kPts; i++) { ones[i] = 1.0f; h[i] = 0.0f; }
                        run.run_node(0, ones, 1.0f, h);
                    }
                    for (uint32_t c = 0; c + 1 < nc; c++) p[c] += tc[c];
                }
                p[nc - 1] += group_mean[g];
                p[nc - 1] += bias[g];
            }
        }
    }
}

void rc_pred_leaf(void* mp, const float* X, uint64_t n, float* out, int32_t nthread) {  // explain.rs:690-701
    const Model& m = *(Model*)mp;
    const uint32_t F = m.n_features, T = (uint32_t)m.trees.size();
    int nth = n_threads(nthread);
#pragma omp parallel for schedule(static) num_threads(nth)
    for (int64_t r = 0; r < (int64_t)n; r++) {
        const float* x = X + (size_t)r * F;
        for (uint32_t t = 0; t < T; t++) {
            const std::vector<Node>& nodes = m.trees[t].nodes;
            size_t i = 0;
            while (!nodes[i].is_leaf) i = node_goes_left(nodes[i], x[nodes[i].feat]) ? (size_t)nodes[i].left : (size_t)nodes[i].right;
            out[(size_t)r * T + t] = (float)i;
        }
    }
}

void rc_pred_approx(void* mp, const float* X, uint64_t n, float* out, int32_t nthread) {  // explain.rs:729-760 saabas_row
    const Model& m = *(Model*)mp;
    const uint32_t F = m.n_features, nc = F + 1;
    std::vector<std::vector<float>> means(m.trees.size());
    for (size_t t = 0; t < m.trees.size(); t++) {  // explain.rs:515-525
        means[t].assign(m.trees[t].nodes.size(), 0.0f);
        fill_node_means(m.trees[t].nodes, 0, means[t]);
    }
    const float bias = base_margin(m.objective, m.base_score);
    int nth = n_threads(nthread);
#pragma omp parallel num_threads(nth)
    {
        std::vector<float> tc(nc);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < (int64_t)n; r++) {
            const float* x = X + (size_t)r * F;
            float* p = out + (size_t)r * nc;
            for (uint32_t c = 0; c < nc; c++) p[c] = 0.0f;
            for (size_t t = 0; t < m.trees.size(); t++) {
                std::fill(tc.begin(), tc.end(), 0.0f);
                const std::vector<Node>& nodes = m.trees[t].nodes;
                const std::vector<float>& mv = means[t];
                float node_value = mv[0];
                tc[nc - 1] += node_value;
                if (!nodes[0].is_leaf) {
                    size_t idx = 0;
                    uint32_t split = 0;
                    while (!nodes[idx].is_leaf) {
                        const Node& nd = nodes[idx];
                        split = nd.feat;
                        idx = node_goes_left(nd, x[split]) ? (size_t)nd.left : (size_t)nd.right;
                        const float nv = mv[idx];
                        tc[split] += nv - node_value;
                        node_value = nv;
                    }
                    tc[split] += nodes[idx].leaf - node_value;
                }
                for (uint32_t c = 0; c < nc; c++) p[c] += tc[c];
            }
            p[nc - 1] += bias;
        }
    }
}

void rc_pred_interactions(void* mp, const float* X, uint64_t n, float* out, int32_t nthread) {  // explain.rs:762-805
    const Model& m = *(Model*)mp;
    const uint32_t F = m.n_features, nc = F + 1;
    double sum = 0.0;
    for (const Tree& t : m.trees) sum += root_mean(t.nodes, 0);
    const float root_mean_f = (float)sum;
    const float bias = base_margin(m.objective, m.base_score);
    const Rule& R = rule();
    int nth = n_threads(nthread);
#pragma omp parallel num_threads(nth)
    {
        std::vector<float> path_prob(F, kUnseen), diag(nc);
        std::vector<std::pair<uint32_t, float>> path;
#pragma omp for schedule(dynamic, 4)
        for (int64_t r = 0; r < (int64_t)n; r++) {
            const float* x = X + (size_t)r * F;
            float* matrix = out + (size_t)r * nc * nc;
            for (size_t c = 0; c < (size_t)nc * nc; c++) matrix[c] = 0.0f;
            std::fill(diag.begin(), diag.end(), 0.0f);
            for (const Tree& t : m.trees) {
                path.clear();
                if (t.nodes[0].is_leaf) continue;
                InteractionRunner run{t.nodes, x, R, path_prob.data(), path, diag.data(), matrix, nc};
                float ones[kPts], h[kPts];
                for (int i = 0; i < kPts; i++) { ones[i] = 1.0f; h[i] = 0.0f; }
                run.run_node(0, ones, 1.0f, h);
            }
            diag[nc - 1] += root_mean_f;
            diag[nc - 1] += bias;
            for (uint32_t a = 0; a < nc; a++)  // symmetric: the mean of the two directions
                for (uint32_t b = a + 1; b < nc; b++) {
                    const float sym = 0.5f * (matrix[a * nc + b] + matrix[b * nc + a]);
                    matrix[a * nc + b] = sym;
                    matrix[b * nc + a] = sym;
                }
            for (uint32_t a = 0; a < nc; a++) {  // diagonal: the additive value minus the row's interactions
                float value = diag[a];
                for (uint32_t b = 0; b < nc; b++)
                    if (b != a) value -= matrix[a * nc + b];
                matrix[a * nc + a] = value;
            }
        }
    }
}

int64_t rc_sketch(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                  const uint8_t* categorical, float* cuts, uint32_t* offsets, uint64_t cap, int32_t nthread) {
    Cuts c = sketch_cuts(X, n, F, max_bin, w, categorical, n_threads(nthread));
    if (c.values.size() > cap) return -1;
    std::memcpy(cuts, c.values.data(), c.values.size() * sizeof(float));
    std::memcpy(offsets, c.offsets.data(), c.offsets.size() * sizeof(uint32_t));
    return (int64_t)c.values.size();
}

void rc_quantize(const float* X, uint64_t n, uint32_t F, const float* cuts, const uint32_t* offsets,
                 const uint8_t* categorical, uint16_t* out) {
    Cuts c;
    c.offsets.assign(offsets, offsets + F + 1);
    c.values.assign(cuts, cuts + offsets[F]);
    if (categorical) c.cat.assign(categorical, categorical + F);
    std::vector<uint16_t> v;
    quantize_cols(X, n, F, c, v, n_threads(0));
    std::memcpy(out, v.data(), v.size() * sizeof(uint16_t));
}

int rc_quantizer(const float* gpair, uint64_t n, uint64_t n_rows, double* scales) {
    double mg = 0, mh = 0;
    for (uint64_t i = 0; i < n; i++) {
        mg = std::max(mg, finite_abs(gpair[2 * i]));
        mh = std::max(mh, finite_abs(gpair[2 * i + 1]));
    }
    if (!std::isfinite(mg) || !std::isfinite(mh)) return -1;
    scales[0] = pow2_scale(mg, n_rows);
    scales[1] = pow2_scale(mh, n_rows);
    return 0;
}

void rc_pow2_scales(const float* max_abs, uint64_t count, uint64_t n_rows, double* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)count; i++) out[i] = pow2_scale((double)max_abs[i], n_rows);
}

// Sum modulo 2^64 of the SplitMix64 finalizer of (scale bits) ^ (b * golden)
// over the f32 bit patterns b in [lo_bits, hi_bits).
uint64_t rc_pow2_scale_digest(uint32_t lo_bits, uint32_t hi_bits, uint64_t n_rows) {
    uint64_t sum = 0;
#pragma omp parallel for schedule(static) reduction(+ : sum)
    for (int64_t b = (int64_t)lo_bits; b < (int64_t)hi_bits; b++) {
        const uint32_t u = (uint32_t)b;
        float f;
        std::memcpy(&f, &u, 4);
        const double s = pow2_scale((double)f, n_rows);
        uint64_t z;
        std::memcpy(&z, &s, 8);
        z ^= (uint64_t)u * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        sum += z ^ (z >> 31);
    }
    return sum;
}

void rc_to_fixed(const float* gpair, uint64_t n, const double* scales, int64_t* out, int64_t* sum) {
    Quantizer q = Quantizer::from_scales(scales[0], scales[1]);
    FX s{0, 0};
    for (uint64_t i = 0; i < n; i++) {
        FX f = q.to_fixed({gpair[2 * i], gpair[2 * i + 1]});
        out[2 * i] = f.g;
        out[2 * i + 1] = f.h;
        s = fx_add(s, f);
    }
    sum[0] = s.g;
    sum[1] = s.h;
}

void rc_hist(const uint16_t* bins, uint64_t n, uint32_t F, const uint32_t* feat_offsets, const uint16_t* missing,
             const int64_t* gpair, const uint32_t* rows, uint64_t n_sel, int64_t* out) {
    FX* h = (FX*)out;
    const FX* g = (const FX*)gpair;
    for (uint32_t f = 0; f < F; f++) {
        const uint16_t* col = bins + (size_t)f * n;
        FX* hf = h + feat_offsets[f];
        uint64_t cnt = rows ? n_sel : n;
        for (uint64_t i = 0; i < cnt; i++) {
            uint32_t r = rows ? rows[i] : (uint32_t)i;
            uint16_t b = col[r];
            if (b == missing[f]) continue;
            hf[b] = fx_add(hf[b], g[r]);
        }
    }
}

void rc_best_split(const int64_t* hist, uint32_t F, const uint32_t* feat_offsets, const int64_t* node_sum,
                   const double* scales, const rc_params* p, float lower, float upper, const uint8_t* enabled,
                   rc_split* out) {
    Params P;
    P.p = *p;
    if (p->monotone) P.mono.assign(p->monotone, p->monotone + F);
    if (p->categorical) P.cat.assign(p->categorical, p->categorical + F);
    Quantizer q = Quantizer::from_scales(scales[0], scales[1]);
    Cand c = best_split((const FX*)hist, F, feat_offsets, FX{node_sum[0], node_sum[1]}, q, P, Bounds{lower, upper},
                        enabled);
    std::memset(out, 0, sizeof(*out));
    out->found = c.found;
    out->feat = c.feat;
    out->bin = c.bin;
    out->missing_left = c.missing_left;
    out->gain = c.gain;
    out->left_g = c.left.g;
    out->left_h = c.left.h;
    out->right_g = c.right.g;
    out->right_h = c.right.h;
    for (size_t i = 0; i < c.cats.size() && i < 8; i++) out->cats[i] = c.cats[i];
}

uint32_t rc_sample_features(uint32_t nf, float rate, uint64_t seed, uint64_t round, uint32_t* out) {
    std::vector<uint32_t> ids = sample_features(nf, rate, seed, round);
    std::copy(ids.begin(), ids.end(), out);
    return (uint32_t)ids.size();
}

void rc_rows_selected(uint64_t n, float rate, uint64_t seed, uint64_t tree, uint8_t* out) {
    const uint64_t th = threshold_for(rate);
    for (uint64_t r = 0; r < n; r++) out[r] = th == UINT64_MAX || (row_hash(r, seed, tree) >> 11) < th;
}

}  // extern "C"
