// Host engine: dataset preparation, the boosting round loop and the model.
//
// Restates the reference's host control (mdai001/FerrisBoost, Rust): the
// weighted quantile sketch and dense quantization (src/data/sketch.rs,
// src/source/dense.rs, src/data/columns.rs), the round loop
// (src/training/mod.rs:1895-2311), column sampling (src/data/colsample.rs),
// row sampling (src/data/subsample.rs) and the XGBoost JSON writer
// (src/model/tree.rs:600-1257).  Per-row and per-bin work runs on the device
// through TrainCtx / ExplainModel (ctx.cu); this file only decides and
// assembles.  Host float steps that must match the reference bit for bit
// (sketch ranks, glibc expf in exact-mode logistic gradients, quantizer
// scales) are compiled with -ffp-contract=off.
#include <algorithm>
#include <charconv>
#include <chrono>
#include <future>
#include <mutex>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <string>
#include <vector>

#include <omp.h>

#include "../../include/fb_engine.h"
#include "ctx.h"
#include "sketch.cuh"

namespace fbe {

// FBGPU_TRACE=1: the wall time of each phase of dataset and booster
// preparation on stderr (phase(name) closes the phase that started at the
// previous call).
struct PhaseTrace {
    const char* what;
    bool on;
    std::chrono::steady_clock::time_point t;
    explicit PhaseTrace(const char* w)
        : what(w), on(std::getenv("FBGPU_TRACE") != nullptr), t(std::chrono::steady_clock::now()) {}
    void operator()(const char* name) {
        if (!on) return;
        const auto now = std::chrono::steady_clock::now();
        std::fprintf(stderr, "[fbgpu] %s %-14s %8.3f ms\n", what, name,
                     std::chrono::duration<double, std::milli>(now - t).count());
        t = now;
    }
};

using fbg::InputError;
thread_local std::string g_err;

// Training features never hold +-inf or f32::MAX: f32::MAX is the upper split
// sentinel (dense.rs:300) and infinities are refused like XGBoost refuses them
// (python/mod.rs:4063-4073 reject_inf).  Prediction input may hold infinities.
const char* const kReservedValue =
    "features cannot be +-inf or the reserved f32::MAX, which marks missing-value split boundaries (use NaN for "
    "missing values; rescale extreme values)";

// ---------------------------------------------------------------- sketch
// sketch.rs:28-435: log-structured merge of compressed weighted summaries.
struct SEntry {
    float v, w, rmin, rmax;
    float rmid() const { return 0.5f * (rmin + rmax); }
};
using Summary = std::vector<SEntry>;

Summary summarize(std::vector<std::pair<float, float>>& buf) {  // sketch.rs:305-329
    std::sort(buf.begin(), buf.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    Summary out;
    out.reserve(buf.size());
    float acc = 0.0f;
    for (size_t i = 0; i < buf.size();) {
        const float v = buf[i].first;
        float w = 0.0f;
        for (; i < buf.size() && buf[i].first == v; i++) w += buf[i].second;
        out.push_back({v, w, acc, acc + w});
        acc += w;
    }
    return out;
}

Summary merge(const Summary& a, const Summary& b) {  // sketch.rs:336-392
    if (a.empty()) return b;
    if (b.empty()) return a;
    Summary m;
    m.reserve(a.size() + b.size());
    size_t i = 0, j = 0;
    float pa = 0.0f, pb = 0.0f;
    while (i < a.size() || j < b.size()) {
        const bool ta = j >= b.size() || (i < a.size() && a[i].v <= b[j].v);
        const SEntry e = ta ? a[i++] : b[j++];
        const float shift = ta ? pb : pa;
        SEntry x{e.v, e.w, e.rmin + shift, e.rmax + shift};
        if (ta) pa = e.rmax; else pb = e.rmax;
        if (!m.empty() && m.back().v == x.v) {
            SEntry& l = m.back();
            l.w += x.w;
            l.rmin = std::min(l.rmin, x.rmin);
            l.rmax = std::max(l.rmax, x.rmax);
        } else {
            m.push_back(x);
        }
    }
    return m;
}

Summary prune(const Summary& e, size_t max_size) {  // sketch.rs:403-435 compress
    const size_t n = e.size();
    if (n <= max_size) return e;
    const float total = e[n - 1].rmax;
    const size_t slots = max_size - 1;
    Summary out;
    out.reserve(max_size);
    out.push_back(e[0]);
    size_t taken = 0;
    for (size_t k = 1; k < slots; k++) {
        const float target = total * (float)k / (float)slots;
        size_t j = taken + 1;
        while (j < n - 1 && e[j].rmid() < target) j++;
        j = std::min(std::max(j, taken + 1), n - 1 - (slots - 1 - k));
        if (j > taken) { out.push_back(e[j]); taken = j; }
    }
    if (taken < n - 1) out.push_back(e[n - 1]);
    return out;
}

std::vector<float> feature_cuts(const fbg::HostMatrix& X, uint64_t n, uint32_t f, uint32_t max_bin,
                                const float* w) {
    const size_t limit = std::max<size_t>((size_t)max_bin * 16, 32);
    std::vector<std::pair<float, float>> buf;
    buf.reserve(limit);
    std::vector<Summary> levels;
    std::vector<char> used;
    auto insert = [&](Summary cur) {  // sketch.rs:161-180
        for (size_t l = 0;; l++) {
            if (l == levels.size()) { levels.push_back(std::move(cur)); used.push_back(1); return; }
            if (!used[l]) { levels[l] = std::move(cur); used[l] = 1; return; }
            Summary ex = std::move(levels[l]);
            levels[l].clear();
            used[l] = 0;
            cur = prune(merge(ex, cur), limit);
        }
    };
    for (uint64_t r = 0; r < n; r++) {  // sketch.rs:128-147 push
        const float v = X.at(r, f);
        const float wt = w ? w[r] : 1.0f;
        if (std::isnan(v) || wt <= 0.0f) continue;
        buf.push_back({v, wt});
        if (buf.size() >= limit) {
            Summary s = prune(summarize(buf), limit);
            buf.clear();
            insert(std::move(s));
        }
    }
    if (!buf.empty()) {
        Summary s = prune(summarize(buf), limit);
        buf.clear();
        insert(std::move(s));
    }
    Summary acc;  // sketch.rs:183-201 collapse
    for (size_t l = 0; l < levels.size(); l++)
        if (used[l]) acc = acc.empty() ? levels[l] : merge(acc, levels[l]);
    if (!acc.empty()) acc = prune(acc, limit);
    std::vector<float> cuts;  // sketch.rs:236-275
    const size_t n_cuts = max_bin >= 1 ? max_bin - 1 : 0;
    if (n_cuts == 0 || acc.empty()) return cuts;
    if (acc.size() <= n_cuts) {
        for (size_t i = 0; i + 1 < acc.size(); i++) {  // sketch.rs:290-302 midpoint
            const float a = acc[i].v, b = acc[i + 1].v;
            const float d = b - a;
            const float m = std::isfinite(d) ? a + d * 0.5f : a * 0.5f + b * 0.5f;
            cuts.push_back(m <= a ? b : m);
        }
        return cuts;
    }
    const float total = acc.back().rmax;
    for (size_t k = 1; k <= n_cuts; k++) {
        const float target = total * (float)k / (float)max_bin;
        size_t idx = std::partition_point(acc.begin(), acc.end(), [&](const SEntry& e) { return e.rmid() < target; }) -
                     acc.begin();
        idx = std::min(idx, acc.size() - 1);
        const float v = acc[idx].v;
        if (cuts.empty() || v > cuts.back()) cuts.push_back(v);
    }
    return cuts;
}

// ---------------------------------------------------------------- dataset
struct Dataset {
    uint64_t n = 0;
    uint32_t F = 0;
    std::vector<float> cuts;
    std::vector<uint32_t> offsets;  // F+1
    std::vector<uint8_t> cat;       // F
    std::vector<uint8_t> width;     // F: bytes per bin
    std::vector<uint8_t> has_nan;   // F: the feature holds a NaN (empty: unknown)
    struct Block {
        std::vector<uint32_t> feats;
        uint32_t width;
        std::vector<uint8_t> data;  // column-major (host datasets)
        std::unique_ptr<fbg::DevMem> dev;  // row records of `stride` bytes (device datasets)
        uint32_t stride = 0;
    };
    std::vector<Block> blocks;
    std::vector<int> feat_block, feat_local;
    int device = -1;  // >= 0: the bins were quantized on this device and live there
    uint32_t n_bins(uint32_t f) const { return offsets[f + 1] - offsets[f] + 1; }
    uint32_t missing(uint32_t f) const { return width[f] == 2 ? 65535u : 255u; }
    float threshold(uint32_t f, uint32_t bin) const {  // tree.rs:991-1000 split_threshold
        const uint32_t nc = offsets[f + 1] - offsets[f];
        if (bin == 0) return -std::numeric_limits<float>::max();
        if (bin > nc) return std::numeric_limits<float>::max();
        return cuts[offsets[f] + bin - 1];
    }
    uint32_t bin_of(uint32_t f, float v) const {  // columns.rs:335-341 find_bin
        if (cat[f]) {  // categorical.rs:360-370 code_to_bin
            const uint32_t nb = n_bins(f);
            if (v >= 0.0f && v < (float)nb) return (uint32_t)v;
            return missing(f) - 1;
        }
        const float* c = cuts.data() + offsets[f];
        return (uint32_t)(std::upper_bound(c, c + (offsets[f + 1] - offsets[f]), v) - c);
    }
};

// bins.rs:58-66 (8 bits unless more bins are needed) and columns.rs:446-461:
// blocks of one width; the device stores every block row-major with a
// 16-byte-padded record, so a block holds at most 64 16-bit or 128 8-bit
// features (128-byte records).
// Bin width per feature (the reference's bins.rs:58-66 picks u8 up to 255
// bins, keeping 255 for missing): one byte up to 255 bins, and also at
// exactly 256 bins when the feature holds no missing value (every byte value
// is then a bin; d.has_nan decides, unknown counts as missing); categorical
// features keep two byte values for missing and invalid codes.
void plan_blocks(Dataset& d) {
    d.width.resize(d.F);
    for (uint32_t f = 0; f < d.F; f++) {
        const uint32_t nb = d.n_bins(f);
        const bool nan = d.has_nan.empty() || d.has_nan[f] != 0;
        const bool wide = d.cat[f] ? nb > 254u : (nb > 256u || (nb == 256u && nan));
        d.width[f] = wide ? 2 : 1;
    }
    d.feat_block.assign(d.F, -1);
    d.feat_local.assign(d.F, -1);
    for (uint32_t w = 1; w <= 2; w++) {
        const uint32_t per = w == 2 ? 64 : 128;
        std::vector<uint32_t> feats;
        for (uint32_t f = 0; f < d.F; f++) if (d.width[f] == w) feats.push_back(f);
        for (size_t i = 0; i < feats.size(); i += per) {
            Dataset::Block b;
            b.width = w;
            b.feats.assign(feats.begin() + i, feats.begin() + std::min(feats.size(), i + per));
            d.blocks.push_back(std::move(b));
        }
    }
    std::sort(d.blocks.begin(), d.blocks.end(), [](const Dataset::Block& a, const Dataset::Block& b) {
        return a.feats[0] < b.feats[0];
    });
    for (size_t bi = 0; bi < d.blocks.size(); bi++) {
        Dataset::Block& b = d.blocks[bi];
        b.stride = ((uint32_t)b.feats.size() * b.width + 15u) / 16u * 16u;
        for (size_t i = 0; i < b.feats.size(); i++) {
            d.feat_block[b.feats[i]] = (int)bi;
            d.feat_local[b.feats[i]] = (int)i;
        }
    }
}

void build_blocks(Dataset& d, const fbg::HostMatrix& X, int nth) {
    // NaN flags of the 256-bin numeric features (the only ones whose width they decide)
    d.has_nan.assign(d.F, 1);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
    for (int64_t f = 0; f < (int64_t)d.F; f++) {
        if (d.cat[f] || d.n_bins((uint32_t)f) != 256u) continue;
        uint8_t any = 0;
        for (uint64_t r = 0; r < d.n && !any; r++) any = std::isnan(X.at(r, (uint32_t)f)) ? 1 : 0;
        d.has_nan[f] = any;
    }
    plan_blocks(d);
    for (Dataset::Block& b : d.blocks) b.data.resize(b.feats.size() * d.n * b.width);
    // dense.rs:288-308 quantize_dense (column-major, NaN -> missing)
    int reserved = 0;
    for (size_t bi = 0; bi < d.blocks.size(); bi++) {
        Dataset::Block& b = d.blocks[bi];
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth) reduction(| : reserved)
        for (int64_t i = 0; i < (int64_t)b.feats.size(); i++) {
            const uint32_t f = b.feats[i];
            const uint32_t miss = d.missing(f);
            for (uint64_t r = 0; r < d.n; r++) {
                const float v = X.at(r, f);
                if (v == std::numeric_limits<float>::max() || std::isinf(v)) reserved = 1;
                const uint32_t bin = std::isnan(v) ? miss : d.bin_of(f, v);
                if (b.width == 2) reinterpret_cast<uint16_t*>(b.data.data())[(size_t)i * d.n + r] = (uint16_t)bin;
                else b.data[(size_t)i * d.n + r] = (uint8_t)bin;
            }
        }
    }
    if (reserved)  // dense.rs:300; python/mod.rs:4063-4073 reject_inf
        throw InputError(kReservedValue);
}

int threads(int32_t nthread) { return nthread > 0 ? nthread : omp_get_max_threads(); }

// Cuts of the listed features (numeric: weighted quantile sketch; categorical:
// 1..max code, sketch.rs:128-136 + categorical.rs:264-266).  Features are
// independent, so row shards on several ranks may each sketch some features.
std::vector<std::vector<float>> sketch_features(const fbg::HostMatrix& X, uint64_t n, uint32_t max_bin,
                                                const float* w, const uint8_t* cat,
                                                const std::vector<uint32_t>& feats, int nth) {
    std::vector<std::vector<float>> per(feats.size());
    std::string bad;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
    for (int64_t i = 0; i < (int64_t)feats.size(); i++) {
        const uint32_t f = feats[i];
        if (cat && cat[f]) {
            int32_t max_code = -1;
            for (uint64_t r = 0; r < n; r++) {
                const float v = X.at(r, f);
                if (std::isnan(v)) continue;
                if (v < 0.0f || v > 65533.0f || v != std::trunc(v)) {
#pragma omp critical
                    bad = "categorical feature #" + std::to_string(f) + " contains an invalid category code";
                    break;
                }
                max_code = std::max(max_code, (int32_t)v);
            }
            for (int32_t k = 1; k <= std::max(max_code, 0); k++) per[i].push_back((float)k);
        } else {
            per[i] = feature_cuts(X, n, f, max_bin, w);
        }
    }
    if (!bad.empty()) throw InputError(bad);
    return per;
}

Dataset* dataset_from_dense(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                            const uint8_t* categorical, int32_t nthread) {
    if (n == 0 || F == 0) throw InputError("training data must have at least one row and one feature");
    if (max_bin == 0 || max_bin > 65535) throw InputError("max_bin must be in 1..=65535");
    if (w)
        for (uint64_t i = 0; i < n; i++)
            if (!std::isfinite(w[i]) || w[i] < 0.0f) throw InputError("sample weights must be finite and non-negative");
    auto d = std::make_unique<Dataset>();
    d->n = n;
    d->F = F;
    d->cat.assign(F, 0);
    if (categorical) for (uint32_t f = 0; f < F; f++) d->cat[f] = categorical[f] ? 1 : 0;
    const int nth = threads(nthread);
    std::vector<uint32_t> all(F);
    for (uint32_t f = 0; f < F; f++) all[f] = f;
    const fbg::HostMatrix hm{X, F, 1};
    std::vector<std::vector<float>> per = sketch_features(hm, n, max_bin, w, d->cat.data(), all, nth);
    d->offsets.push_back(0);
    for (uint32_t f = 0; f < F; f++) {
        d->cuts.insert(d->cuts.end(), per[f].begin(), per[f].end());
        d->offsets.push_back((uint32_t)d->cuts.size());
    }
    build_blocks(*d, hm, nth);
    return d.release();
}

// Cuts of the listed features from the device copy of the rows: the device
// sketch for numeric features (unit weights), the device max-code scan for
// categorical ones (sketch.rs:128-136, categorical.rs:264-266).
std::vector<std::vector<float>> device_sketch(fbg::DeviceMatrix& M, uint32_t max_bin, const uint8_t* cat,
                                              const std::vector<uint32_t>& feats) {
    std::vector<std::vector<float>> per(feats.size());
    std::vector<uint32_t> num, cf, num_i, cf_i;
    for (size_t i = 0; i < feats.size(); i++) {
        const bool c = cat && cat[feats[i]];
        (c ? cf : num).push_back(feats[i]);
        (c ? cf_i : num_i).push_back((uint32_t)i);
    }
    std::vector<std::vector<float>> pn;
    M.numeric_cuts(max_bin, num, pn);
    for (size_t i = 0; i < num.size(); i++) per[num_i[i]] = std::move(pn[i]);
    std::vector<int32_t> mc;
    int64_t bad = -1;
    M.categorical_scan(cf, mc, bad);
    if (bad >= 0)
        throw InputError("categorical feature #" + std::to_string(cf[bad]) + " contains an invalid category code");
    for (size_t i = 0; i < cf.size(); i++)
        for (int32_t k = 1; k <= std::max(mc[i], 0); k++) per[cf_i[i]].push_back((float)k);
    return per;
}

// A stream on `device` for dataset preparation, synchronized and destroyed
// at scope exit.
struct PrepStream {
    cudaStream_t s = nullptr;
    explicit PrepStream(int32_t device) {
        int n_dev = 0;
        if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev)
            throw InputError("device " + std::to_string(device) + " is not a visible CUDA device");
        FB_CUDA_CHECK(cudaSetDevice(device));
        FB_CUDA_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    }
    ~PrepStream() {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
    }
};

// Checks of given cuts (DenseSource::with_cuts): F+1 non-decreasing offsets.
void check_cuts(const uint32_t* offsets, uint32_t F) {
    if (!offsets) throw InputError("cuts need F+1 offsets");
    if (offsets[0] != 0) throw InputError("cut offsets must start at 0");
    for (uint32_t f = 0; f < F; f++)
        if (offsets[f + 1] < offsets[f]) throw InputError("cut offsets must be non-decreasing");
}

// The same dataset as dataset_from_dense / fb_dataset_with_cuts, prepared on
// `device`: the rows are copied to the device once, numeric cuts come from
// the device sketch (unit weights; the host sketch when weights are given,
// since only the order of equal values' weights would differ), categorical
// cuts from a device max-code scan, and the bins are written straight into
// the row records the training context reads, which stay on the device.
Dataset* dataset_on_device(const fbg::HostMatrix& X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                           const uint8_t* categorical, const float* cuts, const uint32_t* offsets, int32_t nthread,
                           int32_t device) {
    if (n == 0 || F == 0) throw InputError("training data must have at least one row and one feature");
    if (!cuts && (max_bin == 0 || max_bin > 65535)) throw InputError("max_bin must be in 1..=65535");
    if (w)
        for (uint64_t i = 0; i < n; i++)
            if (!std::isfinite(w[i]) || w[i] < 0.0f) throw InputError("sample weights must be finite and non-negative");
    PrepStream ps(device);
    const cudaStream_t s = ps.s;
    auto d = std::make_unique<Dataset>();
    d->n = n;
    d->F = F;
    d->device = device;
    d->cat.assign(F, 0);
    if (categorical) for (uint32_t f = 0; f < F; f++) d->cat[f] = categorical[f] ? 1 : 0;
    PhaseTrace phase("dataset");
    fbg::DeviceMatrix M(X, n, F, s, fbe::threads(nthread));
    phase("rows to device");
    if (cuts) {
        check_cuts(offsets, F);
        d->offsets.assign(offsets, offsets + F + 1);
        d->cuts.assign(cuts, cuts + offsets[F]);
    } else {
        std::vector<uint32_t> all(F);
        for (uint32_t f = 0; f < F; f++) all[f] = f;
        std::vector<std::vector<float>> per =
            (w || max_bin * 16ull > fbg::kSketchMaxLimit)
                ? sketch_features(X, n, max_bin, w, d->cat.data(), all, threads(nthread))
                : device_sketch(M, max_bin, d->cat.data(), all);
        d->offsets.push_back(0);
        for (uint32_t f = 0; f < F; f++) {
            d->cuts.insert(d->cuts.end(), per[f].begin(), per[f].end());
            d->offsets.push_back((uint32_t)d->cuts.size());
        }
    }
    phase("sketch");
    d->has_nan = M.nan_features();
    plan_blocks(*d);
    fbg::DevMem d_cuts, d_off, d_cat;
    d_cuts.alloc(std::max<size_t>(d->cuts.size(), 1) * 4);
    d_off.alloc(d->offsets.size() * 4);
    d_cat.alloc(F);
    if (!d->cuts.empty())
        FB_CUDA_CHECK(cudaMemcpyAsync(d_cuts.p, d->cuts.data(), d->cuts.size() * 4, cudaMemcpyHostToDevice, s));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_off.p, d->offsets.data(), d->offsets.size() * 4, cudaMemcpyHostToDevice, s));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_cat.p, d->cat.data(), F, cudaMemcpyHostToDevice, s));
    bool reserved = false;
    for (Dataset::Block& b : d->blocks) {
        b.dev = std::make_unique<fbg::DevMem>();
        b.dev->alloc((size_t)n * b.stride + 16);
        reserved |= M.bin_block(b.feats.data(), (uint32_t)b.feats.size(), b.width, d_cuts.as<float>(),
                                d_off.as<uint32_t>(), d_cat.as<uint8_t>(), b.dev->as<uint8_t>(), b.stride);
    }
    phase("binning");
    if (reserved)  // dense.rs:300; python/mod.rs:4063-4073 reject_inf
        throw InputError(kReservedValue);
    return d.release();
}

// ---------------------------------------------------------------- model
struct Node {
    int32_t left = -1, right = -1;
    uint32_t feat = 0;
    float cond = 0.0f;
    bool default_left = false;
    float leaf = 0.0f;
    bool is_leaf = true;
    bool is_cat = false;
    float gain = 0.0f;
    float hess = 0.0f;
    std::vector<uint32_t> cats;
};
struct Tree {
    std::vector<Node> nodes;
};
struct Model {
    std::vector<Tree> trees;
    float base_score = 0.5f;
    int objective = 1;                 // 0 reg:squarederror, 1 binary:logistic, 2 multi:softprob, 3 multi:softmax
    uint32_t n_features = 0;
    float scale_pos_weight = 1.0f;
    std::vector<uint8_t> feature_types;
    std::vector<float> class_margins;  // multiclass: one base margin per class (tree.rs:260); tree t is class t % K
    std::unique_ptr<fbgpu_model> dev;  // device copy of all trees (prediction / SHAP / leaf indices)
    std::vector<std::unique_ptr<fbgpu_model>> dev_class;  // multiclass: class k's trees, its base margin
    int dev_device = -1;
    size_t dev_trees = 0;
    uint32_t outputs() const { return class_margins.empty() ? 1u : (uint32_t)class_margins.size(); }
};

float base_margin(int objective, float base_score) {  // objective.rs:368-399
    if (objective == 1) {
        const float x = std::min(std::max(base_score, 1e-6f), 1.0f - 1e-6f);
        return -std::log(1.0f / x - 1.0f);
    }
    return base_score;
}

// Shortest round-trip digits of an f32 (the digit string serde_json's ryu and
// Rust's Display both start from) and its decimal exponent.
void shortest(float v, std::string& digits, int& kk) {
    char buf[64];
    auto r = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::scientific);
    std::string s(buf, r.ptr);
    const size_t e = s.find('e');
    digits.clear();
    for (size_t i = 0; i < e; i++) if (s[i] >= '0' && s[i] <= '9') digits.push_back(s[i]);
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    kk = std::atoi(s.c_str() + e + 1) + 1;
}

std::string json_f32(float v) {  // serde_json f32 (ryu layout)
    if (!std::isfinite(v)) return "null";
    std::string o;
    if (std::signbit(v)) { o.push_back('-'); v = -v; }
    if (v == 0.0f) return o + "0.0";
    std::string d;
    int kk;
    shortest(v, d, kk);
    const int len = (int)d.size(), k = kk - len;
    if (0 <= k && kk <= 13) o += d + std::string((size_t)(kk - len), '0') + ".0";
    else if (0 < kk && kk <= 13) o += d.substr(0, kk) + "." + d.substr(kk);
    else if (-6 < kk && kk <= 0) o += "0." + std::string((size_t)(-kk), '0') + d;
    else if (len == 1) o += d + "e" + std::to_string(kk - 1);
    else o += d.substr(0, 1) + "." + d.substr(1) + "e" + std::to_string(kk - 1);
    return o;
}

std::string display_f32(float v) {  // Rust Display for f32
    if (std::isnan(v)) return "NaN";
    std::string o;
    if (std::signbit(v)) { o.push_back('-'); v = -v; }
    if (std::isinf(v)) return o + "inf";
    if (v == 0.0f) return o + "0";
    std::string d;
    int kk;
    shortest(v, d, kk);
    const int len = (int)d.size();
    if (kk <= 0) o += "0." + std::string((size_t)(-kk), '0') + d;
    else if (kk >= len) o += d + std::string((size_t)(kk - len), '0');
    else o += d.substr(0, kk) + "." + d.substr(kk);
    return o;
}

static void json_iarr(std::string& o, const std::vector<int64_t>& v) {
    o.push_back('[');
    for (size_t i = 0; i < v.size(); i++) { if (i) o.push_back(','); o += std::to_string(v[i]); }
    o.push_back(']');
}
static void json_farr(std::string& o, const std::vector<float>& v) {
    o.push_back('[');
    for (size_t i = 0; i < v.size(); i++) { if (i) o.push_back(','); o += json_f32(v[i]); }
    o.push_back(']');
}

// One tree's JSON object (tree.rs:600-750, serde field order of tree.rs:1167-1257).
static std::string tree_json(const Model& m, size_t ti) {
    const std::vector<Node>& N = m.trees[ti].nodes;
    const size_t nn = N.size();
    std::string o;
    o.reserve(64 + nn * 96);
    std::vector<float> bw(nn), lc(nn), sc(nn), sh(nn);
    std::vector<int64_t> dl(nn), lch(nn), rch(nn), par(nn, 2147483647), si(nn), st(nn, 0), cats, cnodes, cseg, csz;
    for (size_t i = 0; i < nn; i++) {
        const Node& nd = N[i];
        lch[i] = nd.left; rch[i] = nd.right; dl[i] = nd.default_left; lc[i] = nd.gain; sh[i] = nd.hess;
        if (nd.is_leaf) { sc[i] = nd.leaf; si[i] = 0; bw[i] = nd.leaf; continue; }
        sc[i] = nd.cond; si[i] = nd.feat; bw[i] = 0.0f;
        par[nd.left] = (int64_t)i; par[nd.right] = (int64_t)i;
        if (nd.is_cat) {
            st[i] = 1;
            cnodes.push_back((int64_t)i);
            cseg.push_back((int64_t)cats.size());
            int64_t c = 0;
            for (size_t w = 0; w < nd.cats.size(); w++)
                for (int b = 0; b < 32; b++)
                    if ((nd.cats[w] >> b) & 1u) { cats.push_back((int64_t)(w * 32 + b)); c++; }
            csz.push_back(c);
        }
    }
    o += "{\"base_weights\":"; json_farr(o, bw);
    o += ",\"categories\":"; json_iarr(o, cats);
    o += ",\"categories_nodes\":"; json_iarr(o, cnodes);
    o += ",\"categories_segments\":"; json_iarr(o, cseg);
    o += ",\"categories_sizes\":"; json_iarr(o, csz);
    o += ",\"default_left\":"; json_iarr(o, dl);
    o += ",\"id\":" + std::to_string(ti);
    o += ",\"left_children\":"; json_iarr(o, lch);
    o += ",\"loss_changes\":"; json_farr(o, lc);
    o += ",\"parents\":"; json_iarr(o, par);
    o += ",\"right_children\":"; json_iarr(o, rch);
    o += ",\"split_conditions\":"; json_farr(o, sc);
    o += ",\"split_indices\":"; json_iarr(o, si);
    o += ",\"split_type\":"; json_iarr(o, st);
    o += ",\"sum_hessian\":"; json_farr(o, sh);
    o += ",\"tree_param\":{\"num_deleted\":\"0\",\"num_feature\":\"" + std::to_string(m.n_features) +
         "\",\"num_nodes\":\"" + std::to_string(nn) + "\",\"size_leaf_vector\":\"1\"}}";
    return o;
}

std::string model_json(const Model& m) {  // tree.rs:600-750, serde field order of tree.rs:1167-1257
    const size_t nt = m.trees.size(), K = m.outputs();
    // the trees' objects are independent: formatted in parallel, joined in order
    std::vector<std::string> parts(nt);
#pragma omp parallel for schedule(dynamic, 4) if (nt >= 16)
    for (int64_t ti = 0; ti < (int64_t)nt; ti++) parts[ti] = tree_json(m, (size_t)ti);
    size_t total = 1024;
    for (const std::string& t : parts) total += t.size() + 1;
    std::string o;
    o.reserve(total + 16 * nt);
    o += "{\"version\":[2,0,0],\"learner\":{\"attributes\":{},\"feature_names\":[],\"feature_types\":[";
    bool any = std::any_of(m.feature_types.begin(), m.feature_types.end(), [](uint8_t c) { return c != 0; });
    if (any)
        for (uint32_t f = 0; f < m.n_features; f++) {
            if (f) o.push_back(',');
            o += m.feature_types[f] ? "\"c\"" : "\"q\"";
        }
    o += "],\"gradient_booster\":{\"name\":\"gbtree\",\"model\":{\"gbtree_model_param\":{\"num_trees\":\"" +
         std::to_string(nt) + "\",\"num_parallel_tree\":\"1\"},\"iteration_indptr\":[";
    // tree.rs:688-697: K trees per round, tree t belongs to output t % K
    for (size_t i = 0; i < nt; i += K) { o += std::to_string(i); o.push_back(','); }
    o += std::to_string(nt);
    o += "],\"tree_info\":[";
    for (size_t i = 0; i < nt; i++) { if (i) o.push_back(','); o += std::to_string(i % K); }
    o += "],\"trees\":[";
    for (size_t ti = 0; ti < nt; ti++) {
        if (ti) o.push_back(',');
        o += parts[ti];
    }
    std::string base = display_f32(m.base_score);
    if (!m.class_margins.empty()) {  // tree.rs:704-720: the vector form "[a,b,c]", margin space
        base = "[";
        for (size_t k = 0; k < K; k++) { if (k) base.push_back(','); base += display_f32(m.class_margins[k]); }
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
        o += "\",\"reg_loss_param\":{\"scale_pos_weight\":\"" + display_f32(m.scale_pos_weight) + "\"}}}}";
    }
    return o;
}

// The device copy of trees cls, cls + step, cls + 2 step, ... (all trees:
// cls = 0, step = 1) with the given base margin.
std::unique_ptr<fbgpu_model> upload_trees(const Model& m, int device, size_t cls, size_t step, float bias) {
    std::vector<uint32_t> off{0}, feat, coff, clen, words;
    std::vector<int32_t> left, right;
    std::vector<float> val, hess;
    std::vector<uint8_t> flags;
    for (size_t ti = cls; ti < m.trees.size(); ti += step) {
        const Tree& t = m.trees[ti];
        for (const Node& nd : t.nodes) {
            left.push_back(nd.left); right.push_back(nd.right); feat.push_back(nd.feat);
            val.push_back(nd.is_leaf ? nd.leaf : nd.cond); hess.push_back(nd.hess);
            flags.push_back((uint8_t)((nd.is_leaf ? 1 : 0) | (nd.default_left ? 2 : 0) | (nd.is_cat ? 4 : 0)));
            coff.push_back((uint32_t)words.size());
            clen.push_back(nd.is_cat ? (uint32_t)nd.cats.size() : 0u);
            if (nd.is_cat) words.insert(words.end(), nd.cats.begin(), nd.cats.end());
        }
        off.push_back((uint32_t)left.size());
    }
    return std::unique_ptr<fbgpu_model>(new fbgpu_model(device, m.n_features, (uint32_t)(off.size() - 1), off.data(),
                                                        left.data(), right.data(), feat.data(), val.data(),
                                                        flags.data(), hess.data(), coff.data(), clen.data(),
                                                        words.data(), words.size(), bias));
}

void ensure_device(Model& m, int device) {
    if (m.dev && m.dev_device == device && m.dev_trees == m.trees.size()) return;
    m.dev = upload_trees(m, device, 0, 1, m.class_margins.empty() ? base_margin(m.objective, m.base_score) : 0.0f);
    m.dev_class.clear();
    for (size_t k = 0; k < m.class_margins.size(); k++)
        m.dev_class.push_back(upload_trees(m, device, k, m.class_margins.size(), m.class_margins[k]));
    m.dev_device = device;
    m.dev_trees = m.trees.size();
}

fbg::ExplainModel& device_model(Model& m, int device) {
    ensure_device(m, device);
    return m.dev->impl;
}

// Per-class outputs of a multiclass model (tree.rs:468-480 predict_margins_upto,
// explain.rs:704-727 one group per class): the rows go to the device once;
// class k's device model writes `width` values per row into a device block,
// copied with a pitch into out[row][k][..].
template <class Fn>
void per_class(Model& m, int device, const float* X, uint64_t n, size_t width, float* out, Fn&& run) {
    ensure_device(m, device);
    const size_t K = m.class_margins.size();
    if (n == 0) return;
    FB_CUDA_CHECK(cudaSetDevice(device));
    fbg::DevMem xd, od;
    xd.alloc(n * m.n_features * sizeof(float));
    od.alloc(n * width * sizeof(float));
    // The class models run on their own non-blocking streams, which do not
    // wait for the legacy default stream, and a plain cudaMemcpy from pageable
    // memory may return before its DMA has landed.  So the rows go up on the
    // first class's stream, and that stream is drained before any class reads
    // them.
    cudaStream_t s0 = m.dev_class[0]->impl.stream();
    FB_CUDA_CHECK(cudaMemcpyAsync(xd.p, X, n * m.n_features * sizeof(float), cudaMemcpyHostToDevice, s0));
    FB_CUDA_CHECK(cudaStreamSynchronize(s0));
    for (size_t k = 0; k < K; k++) {
        fbg::ExplainModel& e = m.dev_class[k]->impl;
        run(e, xd.as<float>(), od.as<float>(), e.stream());
        FB_CUDA_CHECK(cudaMemcpy2DAsync(out + k * width, K * width * sizeof(float), od.p, width * sizeof(float),
                                        width * sizeof(float), n, cudaMemcpyDeviceToHost, e.stream()));
        FB_CUDA_CHECK(cudaStreamSynchronize(e.stream()));
    }
}

// ---------------------------------------------------------------- sampling
inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
uint64_t threshold_for(float rate) {  // subsample.rs:64-73
    if (rate >= 1.0f || !(rate > 0.0f)) return UINT64_MAX;
    return (uint64_t)((double)rate * (double)(1ull << 53));
}
inline bool row_selected(uint64_t row, uint64_t th, uint64_t seed, uint64_t tree) {  // subsample.rs:52-78
    if (th == UINT64_MAX) return true;
    return (mix64(seed ^ rotl(tree * 0x9E3779B97F4A7C15ull, 23) ^ (row * 0xD6E8FEB86659FD93ull)) >> 11) < th;
}
// colsample.rs:29-104: SplitMix64 Fisher-Yates over global feature ids.
std::vector<uint8_t> sample_features(uint32_t nf, float rate, uint64_t seed, uint64_t round) {
    std::vector<uint8_t> en(nf, 1);
    if (rate >= 1.0f) return en;
    double v = std::floor((double)rate * (double)nf);
    uint64_t take = (std::isfinite(v) && v >= 1.0) ? (uint64_t)v : 1;
    take = std::max<uint64_t>(1, std::min<uint64_t>(take, nf));
    if (take >= nf) return en;
    std::vector<uint32_t> ids(nf);
    for (uint32_t i = 0; i < nf; i++) ids[i] = i;
    uint64_t s = seed ^ rotl(round * 0x9E3779B97F4A7C15ull, 17);
    for (uint32_t i = nf - 1; i >= 1; i--) {
        const uint64_t n = (uint64_t)i + 1;
        const uint64_t zone = UINT64_MAX - (UINT64_MAX % n) - 1;
        uint64_t r;
        do { s += 0x9E3779B97F4A7C15ull; r = mix64(s); } while (r > zone);
        std::swap(ids[i], ids[r % n]);
    }
    std::fill(en.begin(), en.end(), 0);
    for (uint64_t i = 0; i < take; i++) en[ids[i]] = 1;
    return en;
}

// ---------------------------------------------------------------- booster
// The f64 sequence a_0 = +0, a_(j+1) = a_j + t (each sum rounded to nearest,
// ties to even), after k steps, without k dependent additions.  Inside one
// binade [2^E, 2^(E+1)) every sum rounds to a multiple of u = 2^(E-52), so
// a_(j+1) = a_j + RN(t / u) u: the increment r is the same at every step,
// except when t / u is an odd multiple of 1/2 (a tie); then it depends on the
// parity of a_j / u until one step has made a_j / u even, and is constant
// after it.  So: single steps until two consecutive increments agree (which
// rules out the parity case), then a jump of s steps of r while every
// unrounded sum stays at least one u below the binade's top; the binade edges
// and subnormal values take single steps.
double repeated_sum(double t, uint64_t k) {
    const bool neg = t < 0.0;
    if (neg) t = -t;  // rounding to nearest is symmetric: the sequence of -t is the negated one
    double a = 0.0;
    while (k > 0) {
        const double n1 = a + t;
        k--;
        if (n1 == a) break;  // a + t rounds back to a: so do all further steps
        a = n1;
        if (k == 0 || !std::isfinite(a) || a < std::numeric_limits<double>::min()) continue;
        const double r1 = (a + t) - a;  // exact: both are multiples of u and r1 <= a
        const double a1 = a + r1;
        const int E = std::ilogb(a);
        if (r1 <= 0.0 || std::ilogb(a1) != E || (a1 + t) - a1 != r1) continue;
        const double u = std::ldexp(1.0, E - 52);
        const double A = a / u, R = r1 / u, T = t / u;      // A, R integers below 2^53
        const double X = 9007199254740991.0 - A;             // 2^53 - 1 - A, exact
        const double sd = std::floor((X - T) / R) - 1.0;     // one fewer than the bound allows, and one
        if (!(sd >= 1.0)) continue;                           // more for the rounding of the division
        const uint64_t s = sd >= (double)k ? k : (uint64_t)sd;
        a = a + (double)s * r1;  // a multiple of u below 2^(E+1): exact
        k -= s;
    }
    return neg ? -a : a;
}

// objective.rs:41-61 label mean (FitInterceptGlmLike), the base_score when
// none is given: a sequential f64 sum in row order.  Labels that take one
// value v besides zero (binary labels) make every term 0 or t = v / n, and
// adding a zero term leaves the sum as it is, so the sum is the k-fold
// sequence of t (k = rows labelled v): repeated_sum gives the same f64 value
// as the row loop without its 11M dependent additions at configs[1].
double label_mean_f64(const float* y, uint64_t n) {
    const double nn = (double)n;
    uint64_t first = 0;
    uint32_t vb = 0;
    for (; first < n; first++) {
        std::memcpy(&vb, y + first, 4);
        if (vb & 0x7fffffffu) break;
    }
    if (first == n) return 0.0;  // every term is a zero
    const float v = y[first];
    if (std::isfinite(v)) {
        int other = 0;
        long long k = 0;
#pragma omp parallel for schedule(static) reduction(+ : k) reduction(| : other)
        for (long long i = (long long)first; i < (long long)n; i++) {
            uint32_t b;
            std::memcpy(&b, y + i, 4);
            k += b == vb;
            other |= (b & 0x7fffffffu) != 0 && b != vb;
        }
        if (!other) return repeated_sum((double)v / nn, (uint64_t)k);
    }
    double acc = 0.0;
    for (uint64_t i = 0; i < n; i++) acc = acc + (double)y[i] / nn;
    return acc;
}

float label_mean(const float* y, const float* w, uint64_t n) {
    if (!w) return (float)label_mean_f64(y, n);
    double sw = 0.0, acc = 0.0;
    for (uint64_t i = 0; i < n; i++) sw = sw + (double)w[i];
    if (sw <= 0.0) return 0.5f;
    for (uint64_t i = 0; i < n; i++) acc = acc + (double)y[i] / sw * (double)w[i];
    return (float)acc;
}

// objective.rs:403-493 initial_base_score for squared error and logistic.
// With |scale_pos_weight - 1| > 1e-6 (compared in f32) it is one Newton step
// from margin 0 over the gradient weights (XGBoost FitIntercept,
// objective.rs:480-493): each row's pair at margin 0 times its gradient weight
// (sample weight, times scale_pos_weight on positives) in f32, summed in f64;
// the step -G / max(H, 1e-6f) rounded to f32 and mapped through the transform
// (sigmoid for logistic, objective.rs:37).  Otherwise the label mean.
float initial_base_score(int objective, const float* y, const float* w, uint64_t n, float spw) {
    if (!(std::fabs(spw - 1.0f) > 1e-6f)) return label_mean(y, w, n);
    double sg = 0.0, sh = 0.0;
    const float s0 = 1.0f / (1.0f + std::exp(-0.0f));
    for (uint64_t i = 0; i < n; i++) {
        const float gw = (w ? w[i] : 1.0f) * (y[i] == 1.0f ? spw : 1.0f);  // mod.rs:5470-5495
        float g = objective == 1 ? s0 - y[i] : 0.0f - y[i];
        float h = objective == 1 ? std::max(s0 * (1.0f - s0), 1e-16f) : 1.0f;
        g = g * gw;
        h = h * gw;
        sg = sg + (double)g;
        sh = sh + (double)h;
    }
    const float m = (float)(-sg / std::max(sh, (double)1e-6f));
    return objective == 1 ? 1.0f / (1.0f + std::exp(-m)) : m;
}

// Row shard of a booster trained on several GPUs (one process per GPU).
struct ShardInfo {
    uint64_t row_offset = 0, n_global = 0;
    const uint8_t* nccl_id = nullptr;
    fbgpu_comm* comm = nullptr;  // a communicator started ahead (fbgpu_comm_begin), else made from nccl_id
    int nranks = 1, rank = 0;
    uint32_t timeout_ms = 0;
};

struct Booster {
    const Dataset* d = nullptr;
    uint64_t row0 = 0, n_global = 0;  // global index of row 0, rows over all ranks
    fb_params p{};
    std::vector<int8_t> mono;
    std::vector<float> labels;  // host copy, kept only for the host-expf logistic rounds
    std::vector<float> grad_w;
    std::unique_ptr<fbg::TrainCtx> ctx;
    Model model;
    uint32_t rounds_done = 0;
    fbg::PinnedMem h_margin, h_exp;
    std::string failed;  // set when a pipelined update failed after the next round was launched
    double t_wall = 0, t_grad = 0, t_tree = 0, t_dev = 0;
    std::vector<int32_t> o_left, o_right;
    std::vector<uint32_t> o_feat, o_bin, o_flags, o_cats;
    std::vector<float> o_gain, o_leaf, o_hess;
};

// objective.rs:1225-1247 initial_class_margins (XGBoost SoftmaxMultiClassObj
// InitEstimation): weighted class counts summed in f32 in row order,
// log((f32)(count / sum_w) + 1e-6) per class, minus their mean taken as
// 0 + v0/K + v1/K + ... in f32.
std::vector<float> initial_class_margins(const float* y, const float* w, uint64_t n, uint32_t K) {
    std::vector<float> bins(K, 0.0f);
    for (uint64_t i = 0; i < n; i++) bins[(size_t)y[i]] += w ? w[i] : 1.0f;
    double sum_w = (double)n;
    if (w) {
        sum_w = 0.0;
        for (uint64_t i = 0; i < n; i++) sum_w += (double)w[i];
    }
    if (sum_w < 1e-6) return std::vector<float>(K, 0.0f);
    const double inv = 1.0 / sum_w;
    std::vector<float> v(K);
    for (uint32_t k = 0; k < K; k++) v[k] = std::log((float)((double)bins[k] * inv) + 1e-6f);
    const float kf = (float)K;
    float mean = 0.0f;
    for (uint32_t k = 0; k < K; k++) mean = mean + v[k] / kf;
    for (uint32_t k = 0; k < K; k++) v[k] = v[k] - mean;
    return v;
}

Booster* booster_create(const Dataset* d, const float* y, const float* w, const fb_params* pp,
                        const ShardInfo& sh = ShardInfo{}) {
    const fb_params& p = *pp;
    if (sh.nranks > 1) {
        if (std::isnan(p.base_score) && !(p.objective >= 2 && p.class_margins))
            throw InputError(p.objective >= 2
                                 ? "a row-sharded multiclass booster needs class_margins (over all rows) or base_score"
                                 : "a row-sharded booster needs base_score (the label mean over all rows)");
        if (!sh.nccl_id && !sh.comm) throw InputError("a row-sharded booster needs an NCCL unique id or communicator");
        if (sh.row_offset + d->n > sh.n_global) throw InputError("row_offset + rows exceeds n_rows_global");
    }
    if (p.objective < 0 || p.objective > 3)
        throw InputError("objective must be reg:squarederror, binary:logistic, multi:softprob or multi:softmax");
    const bool multi = p.objective >= 2;
    if (multi && p.num_class < 2) throw InputError("multi:softprob / multi:softmax need num_class >= 2");
    if (p.max_depth > 14) throw InputError("max_depth must be in 0..=14");
    if (!(p.subsample > 0.0f && p.subsample <= 1.0f)) throw InputError("subsample must be in (0, 1]");
    if (!(p.colsample_bytree > 0.0f && p.colsample_bytree <= 1.0f)) throw InputError("colsample_bytree must be in (0, 1]");
    if (!(p.eta >= 0.0f) || !(p.lambda >= 0.0f) || !(p.gamma >= 0.0f) || !(p.min_child_weight >= 0.0f))
        throw InputError("learning_rate, lambda, gamma and min_child_weight must be finite and non-negative");
    PhaseTrace phase("booster");
    {
        // the label rules, checked in parallel (the first failing rule in this order is reported)
        int bad_finite = 0, bad_range = 0, bad_class = 0;
        const float K = (float)p.num_class;
        const int nth = threads(p.nthread);
#pragma omp parallel for schedule(static) reduction(| : bad_finite, bad_range, bad_class) num_threads(nth)
        for (int64_t i = 0; i < (int64_t)d->n; i++) {
            const float v = y[i];
            bad_finite |= !std::isfinite(v);
            bad_range |= v < 0.0f || v > 1.0f;
            bad_class |= !(v >= 0.0f && v < K && v == std::trunc(v));
        }
        if (bad_finite) throw InputError("labels must all be finite");
        if (p.objective == 1 && bad_range) throw InputError("binary:logistic labels must be in [0, 1]");
        if (multi && bad_class)  // objective.rs:681-688
            throw InputError("multiclass labels must be integers in [0, num_class=" + std::to_string(p.num_class) +
                             ")");
    }
    // the default base score is a sequential f64 sum over the rows (its
    // rounding order is the reference's): computed on a host thread while the
    // device context is set up
    std::future<float> base_later;
    if (!multi && std::isnan(p.base_score))
        base_later = std::async(std::launch::async, [=] {
            return initial_base_score(p.objective, y, w, d->n, p.scale_pos_weight);
        });
    phase("label checks");
    auto b = std::make_unique<Booster>();
    b->d = d;
    b->p = p;
    b->row0 = sh.nranks > 1 ? sh.row_offset : 0;
    b->n_global = sh.nranks > 1 ? sh.n_global : d->n;
    if (p.monotone) b->mono.assign(p.monotone, p.monotone + d->F);
    // mod.rs:5470-5495 gradient weights (sample weight x scale_pos_weight on
    // positives; objective.rs uses_scale_pos_weight: not for multiclass)
    if (p.scale_pos_weight != 1.0f && !multi) {
        b->grad_w.resize(d->n);
        for (uint64_t i = 0; i < d->n; i++) {
            const float wi = w ? w[i] : 1.0f;
            b->grad_w[i] = y[i] == 1.0f ? wi * p.scale_pos_weight : wi;
        }
    } else if (w) {
        b->grad_w.assign(w, w + d->n);
    }
    // objective.rs:41-61 label mean (FitInterceptGlmLike) when base_score is not given
    float base = p.base_score;
    if (multi) {  // mod.rs:1430-1450: per-class margins, the given base_score K times
        if (p.class_margins)
            b->model.class_margins.assign(p.class_margins, p.class_margins + p.num_class);
        else
            b->model.class_margins = std::isnan(base) ? initial_class_margins(y, w, d->n, p.num_class)
                                                      : std::vector<float>(p.num_class, base);
        base = b->model.class_margins[0];
    }
    phase("labels");
    b->model.objective = p.objective;
    b->model.n_features = d->F;
    b->model.scale_pos_weight = p.scale_pos_weight;
    if (std::any_of(d->cat.begin(), d->cat.end(), [](uint8_t c) { return c != 0; })) b->model.feature_types = d->cat;

    fbgpu_config cfg{};
    cfg.device = p.device;
    cfg.n_features = d->F;
    cfg.n_rows = d->n;
    cfg.n_rows_global = b->n_global;
    cfg.row_offset = b->row0;
    cfg.max_depth = p.max_depth;
    cfg.max_leaves = p.max_leaves;
    cfg.gpu_math = p.gpu_math;
    b->ctx.reset(new fbg::TrainCtx(cfg));
    phase("context");
    if (sh.nranks > 1) {
        if (sh.comm) {
            if (sh.comm->impl.nranks != sh.nranks || sh.comm->impl.rank != sh.rank)
                throw InputError("the communicator was started for another rank / world size");
            b->ctx->adopt_comm(sh.comm->impl.share(), sh.nranks, sh.rank);
        } else {
            b->ctx->set_comm(sh.nccl_id, sh.nranks, sh.rank, sh.timeout_ms);
        }
    }
    std::vector<uint32_t> nb(d->F);
    for (uint32_t f = 0; f < d->F; f++) nb[f] = d->n_bins(f);
    b->ctx->set_features(nb.data(), d->width.data(), d->cat.data());
    if (d->device >= 0 && d->device != p.device)
        throw InputError("the dataset was quantized on device " + std::to_string(d->device) +
                         ", the booster runs on device " + std::to_string(p.device));
    for (const Dataset::Block& blk : d->blocks) {
        if (blk.dev)  // device dataset: the context reads its records in place
            b->ctx->adopt_block(blk.feats.data(), (uint32_t)blk.feats.size(), blk.width, blk.dev->as<uint8_t>(),
                                blk.stride);
        else
            b->ctx->upload_block(blk.feats.data(), (uint32_t)blk.feats.size(), blk.width, blk.data.data());
    }
    phase("features, blocks");
    if (base_later.valid()) base = base_later.get();
    if (p.objective == 1 && !(base >= 0.0f && base <= 1.0f))
        throw InputError("logistic base_score is a probability and must be in [0, 1]");
    b->model.base_score = base;
    phase("base score");
    b->ctx->set_labels(y, b->grad_w.empty() ? nullptr : b->grad_w.data(), nullptr, base_margin(p.objective, base));
    if (p.objective == 1 && p.gpu_math != 1 && !b->ctx->has_exact_exp()) {
        // the host-expf rounds read the labels on the host
        b->labels.resize(d->n);
#pragma omp parallel for schedule(static) num_threads(threads(p.nthread))
        for (int64_t c = 0; c < (int64_t)d->n; c += (1 << 18))
            std::memcpy(b->labels.data() + c, y + c, 4 * std::min<uint64_t>(1 << 18, d->n - (uint64_t)c));
    }
    phase("labels upload");
    if (multi) {
        if (p.gpu_math != 1 && !b->ctx->has_exact_exp())
            throw InputError("exact multiclass training needs the verified host-expf table on the device");
        b->ctx->set_outputs(p.num_class, b->model.class_margins.data());
    }
    const uint32_t cap = (2u << p.max_depth);
    b->o_left.resize(cap); b->o_right.resize(cap); b->o_feat.resize(cap); b->o_bin.resize(cap);
    b->o_flags.resize(cap); b->o_cats.resize((size_t)b->ctx->cat_words() * cap); b->o_gain.resize(cap);
    b->o_leaf.resize(cap);
    b->o_hess.resize(cap);
    return b.release();
}

// One boosting round (training/mod.rs:1895-2311).
// A finished device tree (fbgpu_tree_out arrays) as a model tree.
Tree assemble_tree(const Booster& b, const fbgpu_tree_out& out);
fbgpu_tree_params tree_params(const Booster& b);
fbgpu_tree_out tree_out(Booster& b);

// One multiclass round (training/mod.rs:2578-2800): the softmax gradients of
// all K classes from the round's starting margins, then for k = 0..K-1 the
// tree with index round*K + k (which keys row sampling and colsample_bytree)
// on class k's gradient column, adding its leaf values to class k's margins.
void booster_round_multi(Booster& b) {
    const fb_params& p = b.p;
    const uint32_t K = p.num_class;
    const uint64_t th = threshold_for(p.subsample);
    fbg::TrainCtx& ctx = *b.ctx;
    const int fast = p.gpu_math == 1 ? 1 : 0;
    auto t0 = std::chrono::steady_clock::now();
    ctx.softmax_gradients(fast);
    double t_tree = 0;  // tree growth; the rest of the round counts as gradient time
    for (uint32_t k = 0; k < K; k++) {
        const uint64_t tree = (uint64_t)b.rounds_done * K + k;
        ctx.quantize_class(k, th, p.seed, tree, fast);
        std::vector<uint8_t> en = sample_features(b.d->F, p.colsample_bytree, p.seed, tree);
        fbgpu_tree_params tp = tree_params(b);
        fbgpu_tree_out out = tree_out(b);
        ctx.set_pred_column(k);
        auto tb = std::chrono::steady_clock::now();
        ctx.build_tree(tp, p.colsample_bytree < 1.0f ? en.data() : nullptr, &out);
        auto tc = std::chrono::steady_clock::now();
        b.model.trees.push_back(assemble_tree(b, out));
        t_tree += std::chrono::duration<double, std::milli>(tc - tb).count();
    }
    ctx.set_pred_column(0);
    b.rounds_done++;
    b.t_grad += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() - t_tree;
    b.t_tree += t_tree;
}

// One boosting round (training/mod.rs:1895-2311).
void booster_round(Booster& b) {
    const fb_params& p = b.p;
    if (p.objective >= 2) return booster_round_multi(b);
    const uint64_t n = b.d->n;
    const uint32_t round = b.rounds_done;
    const uint64_t th = threshold_for(p.subsample);
    fbg::TrainCtx& ctx = *b.ctx;
    auto t0 = std::chrono::steady_clock::now();
    if (p.gpu_math == 1) {
        ctx.round_device(p.objective, 1, th, p.seed, round, nullptr, nullptr);
    } else if (p.objective == 0 || ctx.has_exact_exp()) {
        // exact squared error, or exact logistic with the device reproduction
        // of the host expf: gradients on the device, scales from the host libm
        ctx.round_device(p.objective, 0, th, p.seed, round, nullptr, nullptr);
    } else {
        // exact logistic: glibc expf on the host, bounds of the f32 gradient,
        // scales with the host libm; the device recomputes the same f32
        // gradient from e and quantizes it (objective.rs:37-39, 519-526).
        b.h_margin.reserve(n * 4);
        b.h_exp.reserve(n * 4);
        float* m = b.h_margin.as<float>();
        float* e = b.h_exp.as<float>();
        ctx.download_margins(m);
        const float* y = b.labels.data();
        const float* gw = b.grad_w.empty() ? nullptr : b.grad_w.data();
        double mg = 0.0, mh = 0.0;
        const int nth = threads(p.nthread);
#pragma omp parallel for schedule(static) reduction(max : mg, mh) num_threads(nth)
        for (int64_t i = 0; i < (int64_t)n; i++) {
            const float ei = std::exp(-m[i]);
            e[i] = ei;
            const float s = 1.0f / (1.0f + ei);
            const float hh = s * (1.0f - s);
            float g = s - y[i];
            float h = hh < 1e-16f ? 1e-16f : hh;
            if (gw) { g = g * gw[i]; h = h * gw[i]; }
            if (!row_selected(b.row0 + (uint64_t)i, th, p.seed, round)) { g = 0.0f; h = 0.0f; }
            mg = std::max(mg, std::isfinite(g) ? std::fabs((double)g) : HUGE_VAL);
            mh = std::max(mh, std::isfinite(h) ? std::fabs((double)h) : HUGE_VAL);
        }
        double m2[2] = {mg, mh};
        ctx.allreduce_max_host(m2, 2);  // global bounds when row-sharded
        mg = m2[0];
        mh = m2[1];
        if (!std::isfinite(mg) || !std::isfinite(mh)) throw InputError("non-finite gradient or Hessian");
        const double sc[2] = {fbg::pow2_scale_host(mg, b.n_global), fbg::pow2_scale_host(mh, b.n_global)};
        ctx.round_from_exp(1, e, th, p.seed, round, sc);
    }
    auto t1 = std::chrono::steady_clock::now();
    std::vector<uint8_t> en = sample_features(b.d->F, p.colsample_bytree, p.seed, round);
    fbgpu_tree_params tp = tree_params(b);
    fbgpu_tree_out out = tree_out(b);
    ctx.build_tree(tp, p.colsample_bytree < 1.0f ? en.data() : nullptr, &out);
    auto t2 = std::chrono::steady_clock::now();
    b.model.trees.push_back(assemble_tree(b, out));
    b.rounds_done++;
    b.t_grad += std::chrono::duration<double, std::milli>(t1 - t0).count();
    b.t_tree += std::chrono::duration<double, std::milli>(t2 - t1).count();
}

// Pipelined rounds: round r+1's gradients and tree are enqueued before tree
// r is read back, so the host's work between rounds (waiting for and reading
// tree r, assembling it, sampling the next round's features, launching) runs
// while the device computes.  It applies when a round needs no host value
// while it runs: gradients and scales on the device (fast mode, squared
// error, or exact logistic with the device expf table), one output, and
// trees that grow without the host (TrainCtx::tree_async).  The model is the
// same: each round reads the margins the previous round's tree left, in
// stream order, and takes its own round index for sampling.
bool pipelinable(const Booster& b) {
    const fb_params& p = b.p;
    if (p.objective >= 2) return false;
    if (!(p.gpu_math == 1 || p.objective == 0 || b.ctx->has_exact_exp())) return false;
    return b.ctx->tree_async(tree_params(b));
}

void launch_round(Booster& b, uint32_t round) {
    const fb_params& p = b.p;
    fbg::TrainCtx& ctx = *b.ctx;
    ctx.round_device(p.objective, p.gpu_math == 1 ? 1 : 0, threshold_for(p.subsample), p.seed, round, nullptr,
                     nullptr);
    // the tree's walk may compute round + 1's gradients from its margins
    ctx.set_next_gradient(p.objective, p.gpu_math == 1 ? 1 : 0, threshold_for(p.subsample), p.seed, round + 1);
    std::vector<uint8_t> en = sample_features(b.d->F, p.colsample_bytree, p.seed, round);
    ctx.build_tree_launch(tree_params(b), p.colsample_bytree < 1.0f ? en.data() : nullptr);
}

void collect_round(Booster& b) {
    fbgpu_tree_out out = tree_out(b);
    b.ctx->build_tree_collect(&out);
    b.model.trees.push_back(assemble_tree(b, out));
    b.rounds_done++;
}

void update_pipelined(Booster& b, uint32_t n_rounds) {
    fbg::TrainCtx& ctx = *b.ctx;
    try {
        for (uint32_t r = 0; r < n_rounds; r++) {
            launch_round(b, b.rounds_done + ctx.trees_in_flight());
            if (ctx.trees_in_flight() == 2) collect_round(b);
        }
        while (ctx.trees_in_flight()) collect_round(b);
    } catch (const std::exception& e) {
        // a round after the failing one may have run: the margins no longer
        // match the model, so the booster takes no further rounds
        b.failed = e.what();
        try {
            ctx.abandon_trees();
        } catch (...) {
        }
        throw;
    }
}

fbgpu_tree_params tree_params(const Booster& b) {
    const fb_params& p = b.p;
    fbgpu_tree_params tp{};
    tp.eta = p.eta; tp.lambda = p.lambda; tp.gamma = p.gamma; tp.min_child_weight = p.min_child_weight;
    tp.alpha = p.alpha; tp.max_delta_step = p.max_delta_step; tp.max_depth = p.max_depth;
    tp.max_leaves = p.max_leaves; tp.max_cat_to_onehot = p.max_cat_to_onehot;
    tp.max_cat_threshold = p.max_cat_threshold; tp.grow_policy = p.grow_policy;
    tp.monotone = b.mono.empty() ? nullptr : b.mono.data();
    return tp;
}

fbgpu_tree_out tree_out(Booster& b) {
    fbgpu_tree_out out{};
    out.capacity = (uint32_t)b.o_left.size();
    out.left = b.o_left.data(); out.right = b.o_right.data(); out.feat = b.o_feat.data(); out.bin = b.o_bin.data();
    out.gain = b.o_gain.data(); out.leaf = b.o_leaf.data(); out.hess = b.o_hess.data(); out.flags = b.o_flags.data();
    const uint32_t W = b.ctx->cat_words();
    if (b.o_cats.size() != (size_t)W * out.capacity) b.o_cats.assign((size_t)W * out.capacity, 0u);
    out.cats = b.o_cats.data();
    out.cat_words = W;
    return out;
}

Tree assemble_tree(const Booster& b, const fbgpu_tree_out& out) {
    Tree t;
    t.nodes.resize(out.n_nodes);
    for (uint32_t i = 0; i < out.n_nodes; i++) {
        Node& nd = t.nodes[i];
        const uint32_t fl = out.flags[i];
        nd.is_leaf = fl & 1u;
        nd.hess = out.hess[i];
        if (nd.is_leaf) { nd.leaf = out.leaf[i]; continue; }
        nd.left = out.left[i]; nd.right = out.right[i]; nd.feat = out.feat[i];
        nd.default_left = (fl & 2u) != 0; nd.gain = out.gain[i]; nd.leaf = 0.0f;
        nd.is_cat = (fl & 4u) != 0;
        if (nd.is_cat) {
            nd.cats.assign(out.cats + (size_t)out.cat_words * i, out.cats + (size_t)out.cat_words * (i + 1));
            while (!nd.cats.empty() && nd.cats.back() == 0) nd.cats.pop_back();
            nd.cond = std::numeric_limits<float>::denorm_min();  // tree.rs:22 CATEGORICAL_SPLIT_COND
        } else {
            nd.cond = b.d->threshold(nd.feat, out.bin[i]);
        }
    }
    return t;
}

template <class F> auto guarded(F&& f, decltype(f()) fail) -> decltype(f()) {
    try {
        return f();
    } catch (const std::exception& e) {
        g_err = e.what();
        return fail;
    }
}

}  // namespace fbe

// ======================================================================= C ABI
struct fb_dataset {
    std::unique_ptr<fbe::Dataset> d;
};
struct fb_booster {
    std::unique_ptr<fbe::Booster> b;
};
struct fb_model : fbe::Model {
    // fb_model_json's text between a size query (buf NULL) and the call that
    // copies it out, so the usual two-call pattern formats the model once
    mutable std::string json_pending;
    mutable std::mutex json_mu;
};

extern "C" {

void fb_default_params(fb_params* p) {  // types.rs:641-686
    std::memset(p, 0, sizeof(*p));
    p->objective = 1;
    p->max_depth = 6;
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

const char* fb_last_error(void) { return fbe::g_err.c_str(); }

fb_dataset* fb_dataset_from_dense(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                                  const uint8_t* categorical, int32_t nthread) {
    return fbe::guarded([&]() -> fb_dataset* {
        auto* out = new fb_dataset();
        out->d.reset(fbe::dataset_from_dense(X, n, F, max_bin, w, categorical, nthread));
        return out;
    }, nullptr);
}

fb_dataset* fb_dataset_with_cuts(const float* X, uint64_t n, uint32_t F, const float* cuts, const uint32_t* offsets,
                                 const uint8_t* categorical, int32_t nthread) {
    return fbe::guarded([&]() -> fb_dataset* {
        std::unique_ptr<fb_dataset> out(new fb_dataset());
        out->d.reset(new fbe::Dataset());
        fbe::Dataset* d = out->d.get();
        d->n = n;
        d->F = F;
        d->offsets.assign(offsets, offsets + F + 1);
        d->cuts.assign(cuts, cuts + offsets[F]);
        d->cat.assign(F, 0);
        if (categorical) for (uint32_t f = 0; f < F; f++) d->cat[f] = categorical[f] ? 1 : 0;
        fbe::build_blocks(*d, fbg::HostMatrix{X, F, 1}, fbe::threads(nthread));
        return out.release();
    }, nullptr);
}

fb_dataset* fb_dataset_on_device(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                                 const uint8_t* categorical, const float* cuts, const uint32_t* offsets,
                                 int32_t nthread, int32_t device) {
    return fbe::guarded([&]() -> fb_dataset* {
        std::unique_ptr<fb_dataset> out(new fb_dataset());
        out->d.reset(fbe::dataset_on_device(fbg::HostMatrix{X, F, 1}, n, F, max_bin, w, categorical, cuts, offsets,
                                            nthread, device));
        return out.release();
    }, nullptr);
}

fb_dataset* fb_dataset_on_device_columns(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                                         const uint8_t* categorical, const float* cuts, const uint32_t* offsets,
                                         int32_t nthread, int32_t device) {
    return fbe::guarded([&]() -> fb_dataset* {
        std::unique_ptr<fb_dataset> out(new fb_dataset());
        out->d.reset(fbe::dataset_on_device(fbg::HostMatrix{X, 1, n}, n, F, max_bin, w, categorical, cuts, offsets,
                                            nthread, device));
        return out.release();
    }, nullptr);
}

int32_t fb_dataset_device(const fb_dataset* h) { return h->d->device; }

int64_t fb_sketch_features_device(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                                  const uint8_t* categorical, const uint32_t* feats, uint32_t n_feats, int32_t nthread,
                                  int32_t device, float* cuts, uint32_t* counts, uint64_t cap) {
    if (w || max_bin * 16ull > fbg::kSketchMaxLimit)
        return fb_sketch_features(X, n, F, max_bin, w, categorical, feats, n_feats, nthread, cuts, counts, cap);
    return fbe::guarded([&]() -> int64_t {
        if (n == 0 || F == 0) throw fbe::InputError("training data must have at least one row and one feature");
        if (max_bin == 0) throw fbe::InputError("max_bin must be in 1..=65535");
        std::vector<uint32_t> fs(feats, feats + n_feats);
        for (uint32_t f : fs)
            if (f >= F) throw fbe::InputError("feature index out of range");
        std::vector<std::vector<float>> per;
        {
            fbe::PrepStream ps(device);
            fbg::DeviceMatrix M(fbg::HostMatrix{X, F, 1}, n, F, ps.s, fbe::threads(nthread));
            per = fbe::device_sketch(M, max_bin, categorical, fs);
        }
        uint64_t total = 0;
        for (size_t i = 0; i < per.size(); i++) total += per[i].size();
        if (total > cap) throw fbe::InputError("cuts capacity is too small: need " + std::to_string(total));
        uint64_t at = 0;
        for (size_t i = 0; i < per.size(); i++) {
            counts[i] = (uint32_t)per[i].size();
            std::memcpy(cuts + at, per[i].data(), 4 * per[i].size());
            at += per[i].size();
        }
        return (int64_t)total;
    }, (int64_t)-1);
}

int64_t fb_sketch_features(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* w,
                           const uint8_t* categorical, const uint32_t* feats, uint32_t n_feats, int32_t nthread,
                           float* cuts, uint32_t* counts, uint64_t cap) {
    return fbe::guarded([&]() -> int64_t {
        if (n == 0 || F == 0) throw fbe::InputError("training data must have at least one row and one feature");
        if (max_bin == 0 || max_bin > 65535) throw fbe::InputError("max_bin must be in 1..=65535");
        if (w)
            for (uint64_t i = 0; i < n; i++)
                if (!std::isfinite(w[i]) || w[i] < 0.0f)
                    throw fbe::InputError("sample weights must be finite and non-negative");
        std::vector<uint32_t> fs(feats, feats + n_feats);
        for (uint32_t f : fs)
            if (f >= F) throw fbe::InputError("feature index out of range");
        auto per = fbe::sketch_features(fbg::HostMatrix{X, F, 1}, n, max_bin, w, categorical, fs, fbe::threads(nthread));
        uint64_t total = 0;
        for (size_t i = 0; i < per.size(); i++) total += per[i].size();
        if (total > cap) throw fbe::InputError("cuts capacity is too small: need " + std::to_string(total));
        uint64_t at = 0;
        for (size_t i = 0; i < per.size(); i++) {
            counts[i] = (uint32_t)per[i].size();
            std::memcpy(cuts + at, per[i].data(), 4 * per[i].size());
            at += per[i].size();
        }
        return (int64_t)total;
    }, (int64_t)-1);
}

float fb_initial_base_score(int32_t objective, const float* labels, const float* weights, uint64_t n,
                            float scale_pos_weight) {
    return fbe::initial_base_score(objective, labels, weights, n, scale_pos_weight);
}

float fb_label_mean(const float* labels, const float* weights, uint64_t n) {
    return fbe::label_mean(labels, weights, n);
}

double fb_label_mean_f64(const float* labels, uint64_t n) { return fbe::label_mean_f64(labels, n); }

int32_t fb_class_margins(const float* labels, const float* weights, uint64_t n, uint32_t K, float* out) {
    return fbe::guarded([&]() -> int32_t {
        if (K < 2) throw fbe::InputError("num_class must be >= 2");
        for (uint64_t i = 0; i < n; i++)
            if (!(labels[i] >= 0.0f && labels[i] < (float)K && labels[i] == std::trunc(labels[i])))
                throw fbe::InputError("multiclass labels must be integers in [0, num_class=" + std::to_string(K) + ")");
        const std::vector<float> v = fbe::initial_class_margins(labels, weights, n, K);
        std::memcpy(out, v.data(), 4ull * K);
        return 0;
    }, 1);
}

void fb_dataset_free(fb_dataset* d) { delete d; }
uint64_t fb_dataset_rows(const fb_dataset* h) { return h->d->n; }

int64_t fb_dataset_cuts(const fb_dataset* h, float* cuts, uint32_t* offsets, uint64_t cap) {
    const fbe::Dataset* d = h->d.get();
    if (offsets) std::memcpy(offsets, d->offsets.data(), 4 * d->offsets.size());
    if (cuts) std::memcpy(cuts, d->cuts.data(), 4 * std::min<uint64_t>(cap, d->cuts.size()));
    return (int64_t)d->cuts.size();
}

int32_t fb_dataset_column(const fb_dataset* h, uint32_t f, uint16_t* out) {
    const fbe::Dataset* d = h->d.get();
    if (f >= d->F) return 1;
    const fbe::Dataset::Block& b = d->blocks[d->feat_block[f]];
    if (b.dev) {  // row records on the device: a strided copy of the feature's bytes
        return fbe::guarded([&]() -> int32_t {
            const size_t lo = (size_t)d->feat_local[f] * b.width;
            std::vector<uint8_t> col((size_t)d->n * b.width);
            FB_CUDA_CHECK(cudaSetDevice(d->device));
            FB_CUDA_CHECK(cudaMemcpy2D(col.data(), b.width, b.dev->as<uint8_t>() + lo, b.stride, b.width, d->n,
                                       cudaMemcpyDeviceToHost));
            for (uint64_t r = 0; r < d->n; r++)
                out[r] = b.width == 2 ? reinterpret_cast<const uint16_t*>(col.data())[r] : col[r];
            return 0;
        }, 2);
    }
    const size_t off = (size_t)d->feat_local[f] * d->n;
    for (uint64_t r = 0; r < d->n; r++)
        out[r] = b.width == 2 ? reinterpret_cast<const uint16_t*>(b.data.data())[off + r] : b.data[off + r];
    return 0;
}

fb_booster* fb_booster_create(const fb_dataset* d, const float* labels, const float* weights, const fb_params* p) {
    return fbe::guarded([&]() -> fb_booster* {
        auto* out = new fb_booster();
        out->b.reset(fbe::booster_create(d->d.get(), labels, weights, p));
        return out;
    }, nullptr);
}

fb_booster* fb_booster_create_sharded(const fb_dataset* shard, const float* labels, const float* weights,
                                      const fb_params* p, uint64_t row_offset, uint64_t n_rows_global,
                                      const uint8_t* nccl_id, int32_t nranks, int32_t rank, uint32_t timeout_ms) {
    return fbe::guarded([&]() -> fb_booster* {
        fbe::ShardInfo sh;
        sh.row_offset = row_offset;
        sh.n_global = n_rows_global;
        sh.nccl_id = nccl_id;
        sh.nranks = nranks;
        sh.rank = rank;
        sh.timeout_ms = timeout_ms;
        if (nranks < 1 || rank < 0 || rank >= nranks) throw fbe::InputError("invalid rank / world size");
        auto* out = new fb_booster();
        std::unique_ptr<fb_booster> guard_out(out);
        out->b.reset(fbe::booster_create(shard->d.get(), labels, weights, p, sh));
        return guard_out.release();
    }, nullptr);
}

fb_booster* fb_booster_create_sharded_comm(const fb_dataset* shard, const float* labels, const float* weights,
                                           const fb_params* p, uint64_t row_offset, uint64_t n_rows_global,
                                           fbgpu_comm* comm, int32_t nranks, int32_t rank) {
    return fbe::guarded([&]() -> fb_booster* {
        fbe::ShardInfo sh;
        sh.row_offset = row_offset;
        sh.n_global = n_rows_global;
        sh.comm = comm;
        sh.nranks = nranks;
        sh.rank = rank;
        if (nranks < 1 || rank < 0 || rank >= nranks) throw fbe::InputError("invalid rank / world size");
        if (nranks > 1 && !comm) throw fbe::InputError("a row-sharded booster needs a communicator");
        auto* out = new fb_booster();
        std::unique_ptr<fb_booster> guard_out(out);
        out->b.reset(fbe::booster_create(shard->d.get(), labels, weights, p, sh));
        return guard_out.release();
    }, nullptr);
}

void fb_booster_free(fb_booster* b) { delete b; }

int32_t fb_booster_update(fb_booster* h, uint32_t n_rounds) {
    fbe::Booster* b = h->b.get();
    return fbe::guarded([&]() -> int32_t {
        if (!b->failed.empty())
            throw fbe::InputError("the booster stopped after an error in an earlier update: " + b->failed);
        b->t_grad = b->t_tree = 0.0;
        b->ctx->reset_stats();
        cudaEvent_t e0, e1;
        FB_CUDA_CHECK(cudaEventCreate(&e0));
        FB_CUDA_CHECK(cudaEventCreate(&e1));
        b->ctx->sync();
        auto t0 = std::chrono::steady_clock::now();
        FB_CUDA_CHECK(cudaEventRecord(e0, b->ctx->stream()));
        if (fbe::pipelinable(*b))
            fbe::update_pipelined(*b, n_rounds);
        else
            for (uint32_t r = 0; r < n_rounds; r++) fbe::booster_round(*b);
        FB_CUDA_CHECK(cudaEventRecord(e1, b->ctx->stream()));
        b->ctx->sync();
        b->t_wall = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        float ms = 0.0f;
        FB_CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        b->t_dev = ms;
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        return 0;
    }, 1);
}

void fb_booster_timing(const fb_booster* h, double* out8) {
    const fbe::Booster* b = h->b.get();
    out8[0] = b->t_wall;
    out8[1] = b->t_grad;
    out8[2] = b->t_tree;
    out8[3] = b->t_dev;
    out8[4] = b->ctx->hist_ms();
    out8[5] = b->ctx->hist_launches();
    out8[6] = b->ctx->hist_bytes();
    out8[7] = (double)b->rounds_done;
}

double fb_booster_collective_ms(const fb_booster* h) { return h->b->ctx->comm_ms(); }
double fb_booster_hist_updates(const fb_booster* h) { return h->b->ctx->hist_updates(); }

void fb_booster_set_stats(fb_booster* h, int32_t on) { h->b->ctx->set_stats(on != 0); }

fb_model* fb_booster_model(fb_booster* h) {
    fbe::Booster* b = h->b.get();
    auto* m = new fb_model();
    m->trees = b->model.trees;
    m->base_score = b->model.base_score;
    m->objective = b->model.objective;
    m->n_features = b->model.n_features;
    m->scale_pos_weight = b->model.scale_pos_weight;
    m->feature_types = b->model.feature_types;
    m->class_margins = b->model.class_margins;
    return m;
}

int32_t fb_booster_margins(fb_booster* h, float* out) {
    return fbe::guarded([&]() -> int32_t { h->b->ctx->download_margins(out); return 0; }, 1);
}

fb_model* fb_train(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const uint8_t* categorical,
                   const fb_params* p, uint32_t n_rounds) {
    fb_dataset* d = fb_dataset_from_dense(X, n, F, p->max_bin, w, categorical, p->nthread);
    if (!d) return nullptr;
    fb_booster* b = fb_booster_create(d, y, w, p);
    if (!b) { fb_dataset_free(d); return nullptr; }
    fb_model* m = nullptr;
    if (fb_booster_update(b, n_rounds) == 0) m = fb_booster_model(b);
    fb_booster_free(b);
    fb_dataset_free(d);
    return m;
}

void fb_model_free(fb_model* m) { delete m; }
uint32_t fb_model_num_trees(const fb_model* m) { return (uint32_t)m->trees.size(); }
uint32_t fb_model_num_features(const fb_model* m) { return m->n_features; }
float fb_model_base_margin(const fb_model* m) { return fbe::base_margin(m->objective, m->base_score); }

int64_t fb_model_json(const fb_model* m, char* buf, int64_t cap) {
    std::lock_guard<std::mutex> lock(m->json_mu);
    if (!buf || cap <= 0) {
        m->json_pending = fbe::model_json(*m);
        return (int64_t)m->json_pending.size();
    }
    std::string s = m->json_pending.empty() ? fbe::model_json(*m) : std::move(m->json_pending);
    m->json_pending.clear();
    std::memcpy(buf, s.data(), (size_t)std::min<int64_t>(cap, (int64_t)s.size()));
    return (int64_t)s.size();
}

fb_model* fb_model_create(uint32_t n_features, int32_t objective, float base_score, float scale_pos_weight,
                          uint32_t num_class, const float* class_margins, const uint8_t* feature_types,
                          uint32_t n_trees, const uint32_t* tree_off, const int32_t* left, const int32_t* right,
                          const uint32_t* feat, const float* cond, const uint8_t* default_left, const float* leaf,
                          const float* gain, const float* hess, const uint8_t* is_cat, const uint32_t* cat_off,
                          const uint32_t* cat_len, const uint32_t* cat_words, uint64_t n_cat_words) {
    return fbe::guarded([&]() -> fb_model* {
        if (n_features == 0) throw fbe::InputError("a model needs at least one feature");
        if (objective < 0 || objective > 3) throw fbe::InputError("unsupported objective code");
        if (objective >= 2 && (num_class < 2 || !class_margins))
            throw fbe::InputError("a multiclass model needs num_class >= 2 and its class margins");
        if (tree_off[0] != 0) throw fbe::InputError("tree offsets must start at 0");
        std::unique_ptr<fb_model> m(new fb_model());
        m->n_features = n_features;
        m->objective = objective;
        m->base_score = base_score;
        m->scale_pos_weight = scale_pos_weight;
        if (objective >= 2) {
            m->class_margins.assign(class_margins, class_margins + num_class);
            m->base_score = class_margins[0];
        }
        if (feature_types) {
            m->feature_types.assign(feature_types, feature_types + n_features);
            if (std::none_of(m->feature_types.begin(), m->feature_types.end(), [](uint8_t c) { return c != 0; }))
                m->feature_types.clear();
        }
        m->trees.resize(n_trees);
        for (uint32_t t = 0; t < n_trees; t++) {
            const uint32_t b = tree_off[t], e = tree_off[t + 1];
            if (e <= b) throw fbe::InputError("tree " + std::to_string(t) + " has no nodes");
            const int32_t nn = (int32_t)(e - b);
            auto& N = m->trees[t].nodes;
            N.resize(nn);
            std::vector<uint8_t> parents(nn, 0);
            auto bad = [&](int32_t i, const std::string& what) {
                return fbe::InputError("tree " + std::to_string(t) + " node " + std::to_string(i) + " " + what);
            };
            for (int32_t i = 0; i < nn; i++) {
                const uint32_t g = b + (uint32_t)i;
                fbe::Node& nd = N[i];
                nd.gain = gain ? gain[g] : 0.0f;
                nd.hess = hess ? hess[g] : 0.0f;
                nd.leaf = leaf[g];
                nd.default_left = default_left[g] != 0;
                if (left[g] < 0) {  // tree.rs:1363-1374: a leaf has no child on either side
                    if (right[g] >= 0) throw bad(i, "has only one child");
                    nd.is_leaf = true;
                    continue;
                }
                // tree.rs:1375-1399: children inside the tree, distinct, each with one parent
                if (right[g] < 0) throw bad(i, "has only one child");
                if (left[g] >= nn || right[g] >= nn || left[g] == right[g])
                    throw bad(i, "has invalid child indices (a child outside the tree, or the same child twice)");
                for (int32_t c : {left[g], right[g]})
                    if (++parents[c] > 1) throw bad(c, "has more than one parent");
                if (feat[g] >= n_features)
                    throw fbe::InputError("tree " + std::to_string(t) + " splits on feature " +
                                          std::to_string(feat[g]) + ", the model has " + std::to_string(n_features));
                nd.is_leaf = false;
                nd.left = left[g];
                nd.right = right[g];
                nd.feat = feat[g];
                nd.cond = cond[g];
                nd.is_cat = is_cat && is_cat[g];
                if (nd.is_cat) {
                    if ((uint64_t)cat_off[g] + cat_len[g] > n_cat_words) throw bad(i, "has a category set out of range");
                    nd.cats.assign(cat_words + cat_off[g], cat_words + cat_off[g] + cat_len[g]);
                    while (!nd.cats.empty() && nd.cats.back() == 0) nd.cats.pop_back();
                }
            }
            // tree.rs:1418-1447: the root has no parent, and a walk from it
            // meets every node exactly once (no cycle, nothing unreachable)
            if (parents[0]) throw bad(0, "(the root) is a child of another node");
            std::vector<uint8_t> seen(nn, 0);
            std::vector<int32_t> stack{0};
            while (!stack.empty()) {
                const int32_t i = stack.back();
                stack.pop_back();
                if (seen[i]) throw fbe::InputError("tree " + std::to_string(t) + " contains a cycle");
                seen[i] = 1;
                if (!N[i].is_leaf) { stack.push_back(N[i].left); stack.push_back(N[i].right); }
            }
            for (int32_t i = 0; i < nn; i++)
                if (!seen[i]) throw bad(i, "is unreachable from the root");
        }
        return m.release();
    }, nullptr);
}

int64_t fb_model_tree(const fb_model* m, uint32_t t, int32_t* left, int32_t* right, uint32_t* feat, float* cond,
                      uint8_t* default_left, float* leaf, uint8_t* is_leaf, float* gain, float* hess, uint32_t* cats) {
    if (t >= m->trees.size()) return -1;
    const auto& N = m->trees[t].nodes;
    for (size_t i = 0; i < N.size(); i++) {
        const fbe::Node& nd = N[i];
        if (left) left[i] = nd.left;
        if (right) right[i] = nd.right;
        if (feat) feat[i] = nd.feat;
        if (cond) cond[i] = nd.cond;
        if (default_left) default_left[i] = nd.default_left;
        if (leaf) leaf[i] = nd.leaf;
        if (is_leaf) is_leaf[i] = nd.is_leaf;
        if (gain) gain[i] = nd.gain;
        if (hess) hess[i] = nd.hess;
        if (cats) for (int w = 0; w < 8; w++) cats[i * 8 + w] = w < (int)nd.cats.size() ? nd.cats[w] : 0u;
    }
    return (int64_t)N.size();
}

int64_t fb_model_node_cats(const fb_model* m, uint32_t t, uint32_t node, uint32_t* out, uint32_t cap) {
    if (t >= m->trees.size() || node >= m->trees[t].nodes.size()) return -1;
    const fbe::Node& nd = m->trees[t].nodes[node];
    if (!nd.is_cat) return 0;
    for (uint32_t w = 0; w < cap && w < nd.cats.size(); w++) out[w] = nd.cats[w];
    return (int64_t)nd.cats.size();
}

int32_t fb_model_predict(fb_model* m, const float* X, uint64_t n, float* out, int32_t device) {
    return fbe::guarded([&]() -> int32_t {
        if (m->outputs() > 1)
            fbe::per_class(*m, device, X, n, 1, out, [&](fbg::ExplainModel& e, const float* xd, float* od,
                                                        cudaStream_t s) { e.predict_device(xd, n, od, s); });
        else
            fbe::device_model(*m, device).predict_host(X, n, out);
        return 0;
    }, 1);
}

uint32_t fb_model_num_outputs(const fb_model* m) { return m->outputs(); }

int32_t fb_model_transform(const fb_model* m, float* margins, uint64_t n, float* classes) {
    return fbe::guarded([&]() -> int32_t {
        const uint32_t K = m->outputs();
        if (m->objective < 2 || K < 2) throw fbe::InputError("fb_model_transform is for multiclass models");
        for (uint64_t r = 0; r < n; r++) {
            float* row = margins + r * K;
            if (m->objective == 3) {  // objective.rs:1324-1333 argmax, first maximum
                uint32_t best = 0;
                for (uint32_t k = 1; k < K; k++)
                    if (row[k] > row[best]) best = k;
                if (classes) classes[r] = (float)best;
            } else {  // objective.rs:1308-1322 softmax_in_place
                float wmax = row[0];
                for (uint32_t k = 1; k < K; k++) wmax = std::fmax(row[k], wmax);
                double wsum = 0.0;
                for (uint32_t k = 0; k < K; k++) {
                    row[k] = std::exp(row[k] - wmax);
                    wsum += (double)row[k];
                }
                const float d = (float)wsum;
                for (uint32_t k = 0; k < K; k++) row[k] /= d;
            }
        }
        return 0;
    }, 1);
}

fbgpu_model* fb_model_device(fb_model* m, int32_t device) {
    return fbe::guarded([&]() -> fbgpu_model* {
        fbe::device_model(*m, device);
        return m->dev.get();
    }, nullptr);
}

int32_t fb_model_shap(fb_model* m, const float* X, uint64_t n, float* out, int32_t device) {
    return fbe::guarded([&]() -> int32_t {
        if (m->outputs() > 1)
            fbe::per_class(*m, device, X, n, (size_t)m->n_features + 1, out,
                           [&](fbg::ExplainModel& e, const float* xd, float* od, cudaStream_t s) {
                               e.shap_device(xd, n, od, s);
                           });
        else
            fbe::device_model(*m, device).shap_host(X, n, out);
        return 0;
    }, 1);
}

int32_t fb_model_explain(fb_model* m, int32_t kind, const float* X, uint64_t n, float* out, int32_t device) {
    return fbe::guarded([&]() -> int32_t {
        if (m->outputs() > 1 && (kind == 1 || kind == 2)) {  // per class: n x K x (F+1) [x (F+1)]
            const size_t nc = (size_t)m->n_features + 1;
            fbe::per_class(*m, device, X, n, kind == 1 ? nc : nc * nc, out,
                           [&](fbg::ExplainModel& e, const float* xd, float* od, cudaStream_t s) {
                               e.explain_device(kind, xd, n, od, s);
                           });
        } else {
            fbe::device_model(*m, device).explain_host(kind, X, n, out);  // leaf indices: all trees in order
        }
        return 0;
    }, 1);
}

}  // extern "C"
