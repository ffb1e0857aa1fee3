// Training context, explanation model and the C ABI of include/fbgpu.h.
#include "ctx.h"

#include <dlfcn.h>
#include <omp.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "fexp.h"

namespace fbg {

namespace {
thread_local std::string g_last_error;
}  // namespace

void noalloc_set_error(const char* msg) { g_last_error = msg; }

namespace {
std::atomic<uint64_t> g_launches{0};
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// ---------------------------------------------------------------- host expf table
namespace {
struct ExpTable {
    bool ok = false;
    std::string why;
    std::vector<std::pair<uint32_t, uint32_t>> entries;  // sorted (input bits, host expf bits)
    std::vector<uint2> slots;
    uint32_t probes = 0;
};

uint32_t host_expf_bits(float x) {
    const float g = expf(x);
    uint32_t b;
    std::memcpy(&b, &g, 4);
    return b;
}

// Loads expf_exceptions.bin (next to this library, or $FBGPU_EXPF_TABLE) and
// checks it against the running host's expf: every listed input, plus 2^21
// pseudo-random inputs, must equal fexp_core corrected by the table.
ExpTable load_exp_table() {
    ExpTable t;
    std::string path;
    if (const char* e = std::getenv("FBGPU_EXPF_TABLE")) {
        path = e;
    } else {
        Dl_info info;
        if (dladdr(reinterpret_cast<void*>(&host_expf_bits), &info) && info.dli_fname) {
            path = info.dli_fname;
            path = path.substr(0, path.find_last_of('/') + 1) + "expf_exceptions.bin";
        }
    }
    FILE* f = path.empty() ? nullptr : std::fopen(path.c_str(), "rb");
    if (!f) { t.why = "exception table not found at " + path; return t; }
    char magic[8];
    uint64_t n = 0;
    bool good = std::fread(magic, 1, 8, f) == 8 && std::memcmp(magic, "FBEXPT01", 8) == 0 &&
                std::fread(&n, 8, 1, f) == 1 && n < (fbx::kExpTableSlots / 2);
    if (good) {
        t.entries.resize(n);
        for (uint64_t i = 0; i < n && good; i++)
            good = std::fread(&t.entries[i].first, 4, 1, f) == 1 && std::fread(&t.entries[i].second, 4, 1, f) == 1;
    }
    std::fclose(f);
    if (!good) { t.why = "malformed exception table " + path; t.entries.clear(); return t; }
    long bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
    for (int64_t i = 0; i < (int64_t)t.entries.size(); i++) {
        float x;
        std::memcpy(&x, &t.entries[i].first, 4);
        if (host_expf_bits(x) != t.entries[i].second) bad++;
    }
#pragma omp parallel for reduction(+ : bad) schedule(static)
    for (int64_t i = 0; i < (1 << 21); i++) {
        uint64_t z = (uint64_t)i * 0x9E3779B97F4A7C15ull + 12345;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z ^= z >> 31;
        uint32_t key = (uint32_t)z;
        if (i & 1) {  // half the sample inside the non-trivial range [-104, 89]
            float x = -104.0f + (float)((z >> 32) % 193000000ull) * 1e-6f;
            std::memcpy(&key, &x, 4);
        }
        float x;
        std::memcpy(&x, &key, 4);
        auto it = std::lower_bound(t.entries.begin(), t.entries.end(), std::make_pair(key, 0u));
        uint32_t want;
        if (it != t.entries.end() && it->first == key) {
            want = it->second;
        } else {
            const float m = fbx::fexp_core(x);
            std::memcpy(&want, &m, 4);
        }
        const uint32_t got = host_expf_bits(x);
        const bool both_nan = std::isnan(x) || (std::isnan(expf(x)));
        if (got != want && !both_nan) bad++;
    }
    if (bad) { t.why = "the exception table does not match this host's expf (" + std::to_string(bad) + " inputs)"; return t; }
    t.slots.assign(fbx::kExpTableSlots, make_uint2(fbx::kEmptyKey, 0u));
    for (const auto& e : t.entries) {
        uint32_t slot = fbx::exp_slot(e.first), len = 1;
        while (t.slots[slot].x != fbx::kEmptyKey) { slot = (slot + 1) & (fbx::kExpTableSlots - 1); len++; }
        t.slots[slot] = make_uint2(e.first, e.second);
        t.probes = std::max(t.probes, len);
    }
    t.probes += 1;  // one more probe sees the empty slot that ends a sequence
    t.ok = true;
    return t;
}

const ExpTable& exp_table() {
    static ExpTable t = load_exp_table();
    return t;
}
}  // namespace

double pow2_scale_host(double max_abs, uint64_t n_rows) {
    if (!(max_abs > 0.0) || !std::isfinite(max_abs)) return 1.0;
    double budget = (double)(1ull << 62) / (double)(n_rows > 0 ? n_rows : 1);
    double raw = budget / max_abs;
    if (!std::isfinite(raw) || raw <= 0.0) return 1.0;
    double l = std::floor(std::log2(raw));
    int k = l >= 2147483647.0 ? 2147483647 : (l <= -2147483648.0 ? (-2147483647 - 1) : (int)l);
    k = std::min(1000, std::max(-1000, k));
    return std::ldexp(1.0, k);
}

std::vector<fbx::ScaleExc> build_scale_exceptions(uint64_t n_rows) {
    // max_abs = budget / 2^k makes raw exactly 2^k; the f32 values around it
    // are the only ones whose raw can sit just below a power of two
    const double budget = fbx::scale_budget(n_rows);
    const int e = std::ilogb(budget);
    std::vector<fbx::ScaleExc> out;
    for (int k = e - 131; k <= e + 151; k++) {
        const float c = (float)std::ldexp(budget, -k);
        if (!std::isfinite(c)) continue;
        float lo = c;
        for (int i = 0; i < 3 && lo > 0.0f; i++) lo = std::nextafter(lo, 0.0f);
        if (!(lo > 0.0f)) lo = std::nextafter(0.0f, 1.0f);
        float f = lo;
        for (int i = 0; i < 7 && std::isfinite(f); i++, f = std::nextafter(f, INFINITY)) {
            const double m = (double)f;
            const double host = pow2_scale_host(m, n_rows);
            if (host != fbx::scale_of_exp(fbx::scale_exp_ilogb(m, n_rows))) {
                uint64_t bits;
                std::memcpy(&bits, &m, 8);
                out.push_back({bits, std::ilogb(host), 0});
            }
        }
    }
    std::sort(out.begin(), out.end(), [](const fbx::ScaleExc& a, const fbx::ScaleExc& b) { return a.bits < b.bits; });
    out.erase(std::unique(out.begin(), out.end(),
                          [](const fbx::ScaleExc& a, const fbx::ScaleExc& b) { return a.bits == b.bits; }),
              out.end());
    return out;
}

// ======================================================================= TrainCtx
void TrainCtx::set_comm(const uint8_t* unique_id, int nranks, int rank, uint32_t timeout_ms) {
    if (!unique_id) throw InputError("unique_id is null");
    if (nranks < 1 || rank < 0 || rank >= nranks) throw InputError("invalid rank / world size");
    if (comm_) throw InputError("the context already has a communicator");
    if (nranks == 1) return;
    comm_.reset(new NcclComm(unique_id, nranks, rank, cfg_.device, timeout_ms));
    nranks_ = nranks;
    rank_ = rank;
}

void TrainCtx::adopt_comm(std::shared_ptr<NcclComm> comm, int nranks, int rank) {
    if (nranks < 1 || rank < 0 || rank >= nranks) throw InputError("invalid rank / world size");
    if (comm_) throw InputError("the context already has a communicator");
    if (nranks == 1) return;
    comm_ = std::move(comm);
    nranks_ = nranks;
    rank_ = rank;
}

void TrainCtx::allreduce_max_host(double* v, int count) {
    if (!comm_ || count <= 0) return;
    if (count > 8) throw InputError("allreduce_max_host takes at most 8 values");
    for (int i = 0; i < count; i++)
        if (!(v[i] >= 0.0)) throw InputError("allreduce_max_host needs non-negative values");
    if (!comm_scratch_.p) comm_scratch_.alloc(64);
    double* h = h_small_.as<double>();
    std::memcpy(h, v, 8ull * count);
    FB_CUDA_CHECK(cudaMemcpyAsync(comm_scratch_.p, h, 8ull * count, cudaMemcpyHostToDevice, s_));
    allreduce_u64(comm_scratch_.p, count, true);
    FB_CUDA_CHECK(cudaMemcpyAsync(h, comm_scratch_.p, 8ull * count, cudaMemcpyDeviceToHost, s_));
    sync();
    std::memcpy(v, h, 8ull * count);
}

// The root gradient sum of a round, over all ranks.  Unless a caller wants it
// now, it rides along with the root's histogram allreduce (one collective
// fewer per round): build_tree appends it to that buffer.
void TrainCtx::reduce_root_sum(bool now) {
    if (!comm_) return;
    if (now) {
        allreduce_u64(sums_.p, 2, false);
        root_pending_ = false;
    } else {
        root_pending_ = true;
    }
}

void TrainCtx::sync() {
    if (comm_) comm_->sync(s_);
    else FB_CUDA_CHECK(cudaStreamSynchronize(s_));
}

void TrainCtx::allreduce_u64(void* buf, size_t count, bool max_op) {
    if (!comm_ || count == 0) return;
    comm_->allreduce(buf, buf, count, /*u64=*/true, max_op, s_);
}

void TrainCtx::allreduce_u32(const void* src, void* dst, size_t count) {
    if (!comm_ || count == 0) return;
    comm_->allreduce(src, dst, count, /*u64=*/false, false, s_);
}

TrainCtx::TrainCtx(const fbgpu_config& cfg) : cfg_(cfg) {
    if (cfg.n_features == 0) throw InputError("training data must have at least one feature");
    if (cfg.n_rows > 0xffffffffull) throw InputError("a shard holds at most 2^32 - 1 rows (u32 row ids)");
    if (cfg.max_depth > 14) throw InputError("max_depth must be in 0..=14");
    FB_CUDA_CHECK(cudaSetDevice(cfg.device));
    FB_CUDA_CHECK(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking));
    h_small_.reserve(1024);  // words 0..9 round values, 32..63 level stats, 80 the scale error word
    FB_CUDA_CHECK(cudaEventCreate(&ev0_));
    FB_CUDA_CHECK(cudaEventCreate(&ev1_));
    for (ReadSlot& sl : slot_) {
        FB_CUDA_CHECK(cudaEventCreate(&sl.ev0));
        FB_CUDA_CHECK(cudaEventCreate(&sl.ev1));
        FB_CUDA_CHECK(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
        for (auto& e : sl.hev) FB_CUDA_CHECK(cudaEventCreate(&e));
        for (auto& e : sl.hevc) FB_CUDA_CHECK(cudaEventCreate(&e));
    }
    level_stats_.alloc(16 * 16);
    n_ = cfg.n_rows;
    F_ = cfg.n_features;
    if (cfg_.n_rows_global == 0) cfg_.n_rows_global = n_;
    smem_budget_ = cfg.hist_smem_bytes ? (int)cfg.hist_smem_bytes : 200 * 1024;
    feat_block_.assign(F_, -1);
    feat_byte_.assign(F_, 0);
    label_.alloc(n_ * 4);
    weight_.alloc(16);
    pred_.alloc(n_ * 4);
    gpair_f32_.alloc(n_ * 8);
    host_exp_.alloc(n_ * 4);
    fixed_.alloc(n_ * 16);
    sums_.alloc(64);
    FB_CUDA_CHECK(cudaMemsetAsync(sums_.p, 0, 64, s_));
    FB_CUDA_CHECK(cudaMemsetAsync(pred_.p, 0, n_ * 4, s_));
    ensure_tree_buffers(cfg.max_depth, cfg.max_leaves);
    const ExpTable& et = exp_table();
    const char* force = std::getenv("FBGPU_EXACT_EXP");
    if (et.ok && !(force && std::string(force) == "host")) {
        exptab_.alloc(sizeof(uint2) * et.slots.size());
        FB_CUDA_CHECK(cudaMemcpyAsync(exptab_.p, et.slots.data(), sizeof(uint2) * et.slots.size(),
                                      cudaMemcpyHostToDevice, s_));
        exp_probes_ = et.probes;
        FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    }
}

TrainCtx::~TrainCtx() {
    if (comm_ && s_) {
        try {
            comm_->sync(s_);
        } catch (const std::exception&) {
        }
    }
    comm_.reset();
    if (s_) cudaStreamSynchronize(s_);
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    for (auto& slot : tree_exec_)
        for (cudaGraphExec_t& e : slot)
            if (e) cudaGraphExecDestroy(e);
    for (ReadSlot& sl : slot_) {
        for (cudaEvent_t e : {sl.ev0, sl.ev1, sl.done}) if (e) cudaEventDestroy(e);
        for (auto& e : sl.hev) if (e) cudaEventDestroy(e);
        for (auto& e : sl.hevc) if (e) cudaEventDestroy(e);
    }
    if (s_) cudaStreamDestroy(s_);
}

void TrainCtx::set_features(const uint32_t* n_bins, const uint8_t* width, const uint8_t* categorical) {
    nbins_.assign(n_bins, n_bins + F_);
    width_.assign(width, width + F_);
    cat_.assign(F_, 0);
    has_cat_ = false;
    if (categorical) {
        for (uint32_t f = 0; f < F_; f++) {
            cat_[f] = categorical[f] ? 1 : 0;
            has_cat_ |= cat_[f] != 0;
        }
    }
    hoff_.assign(F_ + 1, 0);
    cat_slot_.assign(F_, 0);
    n_cat_ = 0;
    cat_words_ = 8;
    for (uint32_t f = 0; f < F_; f++) {
        if (width_[f] != 1 && width_[f] != 2) throw InputError("bin width must be 1 or 2 bytes");
        if (width_[f] == 1 && nbins_[f] > 256) throw InputError("one-byte bins hold at most 256 bins");
        if (nbins_[f] == 0) throw InputError("a feature has at least one bin");
        if (cat_[f]) {
            // codes 0..65533 (categorical.rs:19-28 MAX_CAT_CODE_WIDE); 65535 is the missing sentinel
            if (nbins_[f] > 65534) throw InputError("a categorical feature has at most 65534 bins (codes 0..65533)");
            cat_slot_[f] = n_cat_++;
            cat_words_ = std::max<uint32_t>(cat_words_, (nbins_[f] + 31) / 32);
        } else if (nbins_[f] > 1024) {
            throw InputError("device split search supports at most 1024 bins per numeric feature");
        }
        hoff_[f + 1] = hoff_[f] + nbins_[f];
    }
    total_bins_ = hoff_[F_];
    d_cat_slot_.alloc(4ull * F_);
    FB_CUDA_CHECK(cudaMemcpyAsync(d_cat_slot_.p, cat_slot_.data(), 4ull * F_, cudaMemcpyHostToDevice, s_));
    last_split_cats_.assign(cat_words_, 0u);
    d_hoff_.alloc(4 * (F_ + 1));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_hoff_.p, hoff_.data(), 4 * (F_ + 1), cudaMemcpyHostToDevice, s_));
    d_cat_.alloc(F_);
    FB_CUDA_CHECK(cudaMemcpyAsync(d_cat_.p, cat_.data(), F_, cudaMemcpyHostToDevice, s_));
    d_enabled_.alloc(F_);
    d_mono_.alloc(F_);
    FB_CUDA_CHECK(cudaMemsetAsync(d_mono_.p, 0, F_, s_));
    d_floc_.alloc(sizeof(FeatLoc) * F_);
    d_floc_rec_.alloc(sizeof(FeatLoc) * F_);
    tiles_valid_ = false;
    buf_depth_ = 0xffffffffu;  // histogram slots and category sets depend on the features
    lg_leaves_ = 0xffffffffu;
    ensure_tree_buffers(cfg_.max_depth, cfg_.max_leaves);
    sync();
}

void TrainCtx::ensure_features() const {
    if (nbins_.empty()) throw InputError("fbgpu_set_features must be called before training");
    for (uint32_t f = 0; f < F_; f++)
        if (feat_block_[f] < 0) throw InputError("feature " + std::to_string(f) + " has no uploaded column block");
}

std::unique_ptr<TrainCtx::Block> TrainCtx::new_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width) {
    if (nbins_.empty()) throw InputError("fbgpu_set_features must be called before fbgpu_upload_block");
    if (width != 1 && width != 2) throw InputError("bin width must be 1 or 2 bytes");
    if (n_feats == 0) throw InputError("a column block holds at least one feature");
    auto b = std::make_unique<Block>();
    b->feats.assign(feat_ids, feat_ids + n_feats);
    for (uint32_t i = 0; i < n_feats; i++) {
        uint32_t f = feat_ids[i];
        if (f >= F_) throw InputError("block feature id out of range");
        if (width_[f] != width) throw InputError("a column block must hold features of its own bin width");
        if (i && f <= feat_ids[i - 1]) throw InputError("block feature ids must be ascending");
        if (feat_block_[f] >= 0) throw InputError("feature uploaded twice");
    }
    b->width = width;
    b->stride = ((n_feats * width + 15) / 16) * 16;
    return b;
}

void TrainCtx::register_block(std::unique_ptr<Block> b) {
    // column-major copy for the partition passes, which read one bin per row
    if (n_ > 0) {
        b->cols.alloc((size_t)n_ * b->feats.size() * b->width);
        launch_records_to_columns((int)b->width, b->base, b->stride, n_, (uint32_t)b->feats.size(), b->cols.as<uint8_t>(),
                                  s_);
        FB_CUDA_CHECK(cudaGetLastError());
    }
    std::vector<FeatLoc> floc(F_), floc_rec(F_);
    const int bi = (int)blocks_.size();
    for (uint32_t i = 0; i < (uint32_t)b->feats.size(); i++) {
        feat_block_[b->feats[i]] = bi;
        feat_byte_[b->feats[i]] = i * b->width;
    }
    blocks_.push_back(std::move(b));
    for (uint32_t f = 0; f < F_; f++) {
        if (feat_block_[f] < 0) { floc[f] = floc_rec[f] = FeatLoc{nullptr, 0, 0, 1, 255}; continue; }
        const Block& blk = *blocks_[feat_block_[f]];
        // the missing sentinel: 65535 / 255, none for a full-range one-byte
        // feature (256 bins: it holds no missing value)
        const uint32_t miss = blk.width == 2 ? 65535u : (nbins_[f] <= 255u ? 255u : 0xffffffffu);
        if (blk.cols.p)
            floc[f] = FeatLoc{blk.cols.as<uint8_t>() + (size_t)(feat_byte_[f] / blk.width) * n_ * blk.width, blk.width,
                              0, blk.width, miss};
        else
            floc[f] = FeatLoc{blk.base, blk.stride, feat_byte_[f], blk.width, miss};
        floc_rec[f] = FeatLoc{blk.base, blk.stride, feat_byte_[f], blk.width, miss};
    }
    FB_CUDA_CHECK(cudaMemcpyAsync(d_floc_.p, floc.data(), sizeof(FeatLoc) * F_, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_floc_rec_.p, floc_rec.data(), sizeof(FeatLoc) * F_, cudaMemcpyHostToDevice, s_));
    sync();
    tiles_valid_ = false;
}

void TrainCtx::adopt_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width, const uint8_t* records,
                           uint32_t stride) {
    auto b = new_block(feat_ids, n_feats, width);
    if (stride != b->stride) throw InputError("row records must be padded to a multiple of 16 bytes");
    if (!records) throw InputError("null row records");
    b->base = records;
    register_block(std::move(b));
}

void TrainCtx::upload_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width, const void* data) {
    auto b = new_block(feat_ids, n_feats, width);
    b->data.alloc((size_t)n_ * b->stride + 16);
    b->base = b->data.as<uint8_t>();
    FB_CUDA_CHECK(cudaMemsetAsync(b->data.p, 0, (size_t)n_ * b->stride + 16, s_));
    // column-major host block -> staging -> row-major records, in row slabs
    const uint64_t slab = std::max<uint64_t>(1, std::min<uint64_t>(n_, (256ull << 20) / ((uint64_t)n_feats * width)));
    DevMem stage;
    stage.alloc(slab * n_feats * width);
    std::vector<uint8_t> host;
    host.resize(slab * n_feats * width);
    const uint8_t* src = static_cast<const uint8_t*>(data);
    for (uint64_t r0 = 0; r0 < n_; r0 += slab) {
        uint64_t rows = std::min(slab, n_ - r0);
        for (uint32_t i = 0; i < n_feats; i++)
            std::memcpy(host.data() + (size_t)i * rows * width, src + ((size_t)i * n_ + r0) * width, rows * width);
        FB_CUDA_CHECK(cudaMemcpyAsync(stage.p, host.data(), rows * n_feats * width, cudaMemcpyHostToDevice, s_));
        launch_transpose((int)width, stage.as<uint8_t>(), b->data.as<uint8_t>(), (uint32_t)rows, n_feats, b->stride,
                         r0, s_);
        sync();
    }
    register_block(std::move(b));
}

void TrainCtx::set_labels(const float* labels, const float* weights, const float* base_rows, float base_margin) {
    next_grad_.set = fused_grad_.set = false;
    FB_CUDA_CHECK(cudaMemcpyAsync(label_.p, labels, n_ * 4, cudaMemcpyHostToDevice, s_));
    has_weight_ = weights != nullptr;
    if (weights) {
        weight_.alloc(n_ * 4);
        FB_CUDA_CHECK(cudaMemcpyAsync(weight_.p, weights, n_ * 4, cudaMemcpyHostToDevice, s_));
    }
    if (base_rows) {
        FB_CUDA_CHECK(cudaMemcpyAsync(pred_.p, base_rows, n_ * 4, cudaMemcpyHostToDevice, s_));
    } else {
        launch_fill(pred_.as<float>(), n_, base_margin, s_);
        FB_CUDA_CHECK(cudaGetLastError());
    }
    sync();
}

GradArgs TrainCtx::grad_args() const {
    GradArgs a{};
    a.n = (uint32_t)n_;
    a.row0 = cfg_.row_offset;
    a.sub_th = ~0ull;
    a.label = label_.as<float>();
    a.weight = has_weight_ ? weight_.as<float>() : nullptr;
    a.pred = pred_.as<float>() + (size_t)pred_col_ * n_;
    a.host_exp = host_exp_.as<float>();
    a.gpair_in = gpair_f32_.as<float>();
    a.gpair_f32 = gpair_f32_.as<float>();
    a.fixed = fixed_.as<Pair>();
    a.sum = sums_.as<unsigned long long>();
    a.maxbits = sums_.as<unsigned long long>() + 2;
    a.scales = reinterpret_cast<const double*>(sums_.as<unsigned long long>() + 4);
    a.exptab = exptab_.p ? exptab_.as<uint2>() : nullptr;
    a.exp_probes = exp_probes_;
    return a;
}

void TrainCtx::upload_and_quantize(const float* gpair, uint64_t th, uint64_t seed, uint64_t tree,
                                   double* scales_out, int64_t* sum_out) {
    FB_CUDA_CHECK(cudaMemcpyAsync(gpair_f32_.p, gpair, n_ * 8, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemsetAsync(sums_.p, 0, 32, s_));
    GradArgs a = grad_args();
    a.sub_th = th; a.sub_seed = seed; a.sub_tree = tree;
    launch_mask_max(a, s_);
    allreduce_u64(a.maxbits, 2, true);
    unsigned long long* mb = h_small_.as<unsigned long long>();
    FB_CUDA_CHECK(cudaMemcpyAsync(mb, sums_.as<unsigned long long>() + 2, 16, cudaMemcpyDeviceToHost, s_));
    sync();
    double mg, mh;
    std::memcpy(&mg, &mb[0], 8);
    std::memcpy(&mh, &mb[1], 8);
    if (!std::isfinite(mg) || !std::isfinite(mh))
        throw InputError("non-finite gradient or Hessian (or invalid bounds); reduce extreme labels, weights, "
                         "base_score or objective parameters");
    double* sc = h_small_.as<double>() + 2;
    sc[0] = pow2_scale_host(mg, cfg_.n_rows_global);
    sc[1] = pow2_scale_host(mh, cfg_.n_rows_global);
    FB_CUDA_CHECK(cudaMemcpyAsync(sums_.as<unsigned long long>() + 4, sc, 16, cudaMemcpyHostToDevice, s_));
    launch_quantize(a, s_);
    reduce_root_sum(sum_out != nullptr);
    if (scales_out) { scales_out[0] = sc[0]; scales_out[1] = sc[1]; }
    int64_t* hs = h_small_.as<int64_t>() + 4;
    FB_CUDA_CHECK(cudaMemcpyAsync(hs, sums_.p, 16, cudaMemcpyDeviceToHost, s_));
    sync();
    if (sum_out) { sum_out[0] = hs[0]; sum_out[1] = hs[1]; }
}

void TrainCtx::upload_fixed(const int64_t* fixed, const double* scales, const int64_t* sum) {
    FB_CUDA_CHECK(cudaMemcpyAsync(fixed_.p, fixed, n_ * 16, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(sums_.p, sum, 16, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(sums_.as<unsigned long long>() + 4, scales, 16, cudaMemcpyHostToDevice, s_));
    sync();
}

void TrainCtx::round_from_exp(int objective, const float* host_exp, uint64_t th, uint64_t seed, uint64_t tree,
                              const double* scales) {
    if (host_exp) FB_CUDA_CHECK(cudaMemcpyAsync(host_exp_.p, host_exp, n_ * 4, cudaMemcpyHostToDevice, s_));
    double* hsc = h_small_.as<double>() + 8;
    hsc[0] = scales[0];
    hsc[1] = scales[1];
    FB_CUDA_CHECK(cudaMemcpyAsync(sums_.as<unsigned long long>() + 4, hsc, 16, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemsetAsync(sums_.p, 0, 16, s_));
    GradArgs a = grad_args();
    a.sub_th = th; a.sub_seed = seed; a.sub_tree = tree;
    a.objective = objective;
    launch_gradient_quantize_exp(a, s_);
    reduce_root_sum(false);
}

void TrainCtx::launch_scales(const unsigned long long* maxbits, bool fast) {
    double* dscales = reinterpret_cast<double*>(sums_.as<unsigned long long>() + 4);
    unsigned long long* err = sums_.as<unsigned long long>() + 6;
    if (fast) {
        launch_device_scales(maxbits, cfg_.n_rows_global, dscales, err, s_);
    } else {
        if (scale_exc_rows_ != cfg_.n_rows_global) {
            const std::vector<fbx::ScaleExc> exc = build_scale_exceptions(cfg_.n_rows_global);
            d_scale_exc_.alloc(sizeof(fbx::ScaleExc) * std::max<size_t>(exc.size(), 1));
            if (!exc.empty())
                FB_CUDA_CHECK(cudaMemcpyAsync(d_scale_exc_.p, exc.data(), sizeof(fbx::ScaleExc) * exc.size(),
                                              cudaMemcpyHostToDevice, s_));
            n_scale_exc_ = (uint32_t)exc.size();
            scale_exc_rows_ = cfg_.n_rows_global;
            sync();  // the host vector goes out of scope
        }
        launch_device_scales_exact(maxbits, cfg_.n_rows_global, d_scale_exc_.as<fbx::ScaleExc>(), n_scale_exc_,
                                   dscales, err, s_);
    }
    scale_err_pending_ = true;
}

void TrainCtx::check_scale_error(const unsigned long long* host_err) {
    if (!scale_err_pending_) return;
    scale_err_pending_ = false;
    if (*host_err) throw InputError("non-finite gradient or Hessian");
}

void TrainCtx::set_next_gradient(int objective, int fast, uint64_t th, uint64_t seed, uint64_t tree) {
    next_grad_.set = K_ == 1 && (objective == 0 || objective == 1) && (fast || objective == 0 || exptab_.p);
    next_grad_.objective = objective;
    next_grad_.fast = fast ? 1 : 0;
    next_grad_.th = th;
    next_grad_.seed = seed;
    next_grad_.tree = tree;
}

void TrainCtx::round_device(int objective, int fast, uint64_t th, uint64_t seed, uint64_t tree, double* scales_out,
                            int64_t* sum_out) {
    // the previous tree's walk already wrote this round's gradient pairs and
    // their bounds (same parameters, margins untouched since)
    const bool done = fused_grad_.same(objective, fast ? 1 : 0, th, seed, tree);
    fused_grad_.set = false;
    FB_CUDA_CHECK(cudaMemsetAsync(sums_.p, 0, done ? 16 : 32, s_));
    GradArgs a = grad_args();
    a.sub_th = th; a.sub_seed = seed; a.sub_tree = tree;
    a.objective = objective;
    if (!fast && objective == 1 && !a.exptab)
        throw InputError("exact logistic gradients on the device need the verified host-expf table; "
                         "use fbgpu_round_from_exp with host exp values");
    if (!done) launch_gradient_max(a, fast ? 1 : (objective == 1 ? 2 : 0), s_);
    allreduce_u64(a.maxbits, 2, true);
    launch_scales(a.maxbits, fast != 0);
    launch_quantize(a, s_);
    reduce_root_sum(sum_out != nullptr);
    read_scales_sum(scales_out, sum_out);
}

// Scales and root sum of the round to the host (when asked for: a sync).
void TrainCtx::read_scales_sum(double* scales_out, int64_t* sum_out) {
    if (!scales_out && !sum_out) return;
    unsigned long long* hs = h_small_.as<unsigned long long>() + 4;
    FB_CUDA_CHECK(cudaMemcpyAsync(hs, sums_.as<unsigned long long>() + 4, 24, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(hs + 3, sums_.p, 16, cudaMemcpyDeviceToHost, s_));
    sync();
    check_scale_error(hs + 2);
    if (scales_out) std::memcpy(scales_out, hs, 16);
    if (sum_out) std::memcpy(sum_out, hs + 3, 16);
}

void TrainCtx::set_outputs(uint32_t K, const float* class_margins) {
    next_grad_.set = fused_grad_.set = false;
    if (K < 2) throw InputError("a multiclass context needs at least 2 classes");
    K_ = K;
    pred_col_ = 0;
    pred_.alloc((size_t)K * n_ * 4);
    gp_multi_.alloc((size_t)K * n_ * 8);
    std::vector<float> v((size_t)K * n_);
    for (uint32_t k = 0; k < K; k++) std::fill(v.begin() + (size_t)k * n_, v.begin() + (size_t)(k + 1) * n_, class_margins[k]);
    FB_CUDA_CHECK(cudaMemcpyAsync(pred_.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice, s_));
    sync();
}

void TrainCtx::softmax_gradients(int fast) {
    if (K_ < 2) throw InputError("softmax gradients need a multiclass context");
    if (!fast && !exptab_.p)
        throw InputError("exact multiclass gradients on the device need the verified host-expf table");
    GradArgs a = grad_args();
    a.pred = pred_.as<float>();
    launch_softmax_gradients(a, K_, gp_multi_.as<float>(), fast, s_);
}

void TrainCtx::quantize_class(uint32_t k, uint64_t th, uint64_t seed, uint64_t tree, int fast, double* scales_out,
                              int64_t* sum_out) {
    FB_CUDA_CHECK(cudaMemsetAsync(sums_.p, 0, 32, s_));
    GradArgs a = grad_args();
    a.sub_th = th; a.sub_seed = seed; a.sub_tree = tree;
    a.gpair_in = gp_multi_.as<float>() + 2ull * k * n_;
    launch_mask_max(a, s_);  // mod.rs:4811-4842 mask_and_bounds
    allreduce_u64(a.maxbits, 2, true);
    launch_scales(a.maxbits, fast != 0);
    launch_quantize(a, s_);
    reduce_root_sum(sum_out != nullptr);
    read_scales_sum(scales_out, sum_out);
}

void TrainCtx::ensure_tree_buffers(uint32_t max_depth, uint32_t max_leaves, bool lossguide) {
    if (max_depth == buf_depth_ && max_leaves == buf_leaves_ && lossguide == buf_lossguide_) return;
    uint64_t lvl = 1ull << max_depth;                 // nodes of the deepest level
    uint64_t split_nodes = max_depth ? (1ull << (max_depth - 1)) : 1;  // deepest split level
    uint64_t acc = max_depth >= 2 ? (1ull << (max_depth - 2)) : 1;
    if (max_leaves) {
        lvl = std::min<uint64_t>(lvl, std::max<uint64_t>(max_leaves, 1));
        split_nodes = std::min<uint64_t>(split_nodes, std::max<uint64_t>(max_leaves, 1));
        acc = std::min<uint64_t>(acc, std::max<uint64_t>(max_leaves, 1));
    }
    uint64_t tree_nodes = (2ull << max_depth) - 1;
    if (max_leaves) tree_nodes = std::min<uint64_t>(tree_nodes, 2ull * max_leaves + 1);
    if (lossguide) {
        // best-first waves (lossguide.cu): up to max_leaves expansions per wave,
        // two evaluated children each; hist_[0] is the histogram pool
        lvl = 2ull * max_leaves + 2;
        split_nodes = 2ull * max_leaves + 4;
        acc = (uint64_t)max_leaves + 1;
        tree_nodes = 2ull * max_leaves + 1;
    }
    max_level_nodes_ = (uint32_t)lvl;
    max_split_nodes_ = (uint32_t)split_nodes;
    max_acc_ = (uint32_t)acc;
    max_tree_nodes_ = (uint32_t)tree_nodes;
    max_chunks_ = ceil_div(std::max<uint64_t>(n_, 1), kChunkRows) + max_level_nodes_ + 1;
    const uint64_t tb = std::max<uint64_t>(total_bins_, 1);
    for (int i = 0; i < 2; i++) {
        rows_[i].alloc(std::max<uint64_t>(n_, 1) * 4);
        nodes_[i].alloc(sizeof(NodeInfo) * lvl);
        acc_list_[i].alloc(4 * (lvl + 1));
        acc_prefix_[i].alloc(8 * (lvl + 2));
        chunk_prefix_[i].alloc(4 * (lvl + 2));
        hist_[i].alloc(lossguide && i == 1 ? 16 : 16 * tb * split_nodes);
    }
    hist_acc_.alloc(16 * tb * acc + 16);  // + the root sum riding on the root's allreduce
    const uint64_t set_bytes = 4ull * cat_words_;
    feat_best_.alloc(sizeof(SplitRec) * split_nodes * F_);
    feat_cats_.alloc(set_bytes * split_nodes * std::max<uint32_t>(n_cat_, 1));
    node_best_.alloc(sizeof(SplitRec) * split_nodes);
    node_cats_.alloc(set_bytes * std::max<uint64_t>(lvl, 1));
    FB_CUDA_CHECK(cudaMemsetAsync(node_cats_.p, 0, node_cats_.bytes, s_));
    split_.alloc(sizeof(SplitDesc) * lvl);
    chunk_left_.alloc(4 * (uint64_t)max_chunks_);
    dirflags_.alloc((uint64_t)max_chunks_ * kPartThreads);
    chunk_off_.alloc(4 * (uint64_t)max_chunks_);
    node_left_.alloc(4 * lvl);
    part_cnt_.alloc(8 * lvl);
    FB_CUDA_CHECK(cudaMemsetAsync(part_cnt_.p, 0, part_cnt_.bytes, s_));
    node_left_global_.alloc(4 * lvl);
    trec_.alloc(sizeof(TreeRec) * tree_nodes);
    tcats_.alloc(set_bytes * tree_nodes);
    state_.alloc(sizeof(TreeState));
    buf_depth_ = max_depth;
    buf_leaves_ = max_leaves;
    buf_lossguide_ = lossguide;
}

// Histogram tiles: the enabled features of every block, grouped per kernel.
// Lane-per-feature tiles take up to 32 features whose [bin][32] planes fit in
// shared memory (features of at most kLpfMaxBins bins); wide tiles take up to
// 8 two-byte features of at most kWideMaxBins bins whose bins lie within 4
// record chunks (the staged kernel with 8 lanes per row); the remaining
// features go to row-per-thread tiles sized by the shared-memory budget.
void TrainCtx::plan_tiles(const uint8_t* enabled, bool rank_major) {
    std::vector<uint8_t> en(F_, 1);
    if (enabled) for (uint32_t f = 0; f < F_; f++) en[f] = enabled[f] ? 1 : 0;
    if (tiles_valid_ && en == last_enabled_ && rank_major == tiles_rank_major_) return;
    // a feature's bin index in the accumulate histograms: its offset, or for
    // the rank-major layout its rank (top 8 bits) and offset in the rank's block
    auto gbin = [&](uint32_t f) -> uint32_t {
        if (!rank_major) return hoff_[f];
        const uint32_t r = feat_rank_[f];
        return (r << 24) | (hoff_[f] - rank_bin_lo_[r]);
    };
    const uint32_t kLpfMaxBins = 440;    // 440 x 32 lanes x 16 B = 220 KiB
    const uint32_t kWideMaxBins = 1024;  // 1028 x 8 lanes x 16 B = 128.5 KiB
    const uint32_t kWideMaxChunks = 4;
    auto is_wide = [&](uint32_t f, uint32_t width) {
        return width == 2 && nbins_[f] > kLpfMaxBins && nbins_[f] <= kWideMaxBins;
    };
    std::vector<TileDesc> gen[2], lpf[2], wide, direct[2];
    std::vector<TileFeat> tf;
    size_t smem_gen = 16, smem_lpf = 16, smem_wide = 16;
    uint32_t max_chunks = 0, max_chunks_wide = 0;
    const uint32_t max_local = (uint32_t)((smem_budget_ - 64 * sizeof(TileFeat)) / 16);
    for (const auto& bp : blocks_) {
        const Block& b = *bp;
        const int wi = (int)b.width - 1;
        const uint32_t miss = b.width == 2 ? 65535u : 255u;
        // lane-per-feature tiles
        TileDesc cur{b.base, b.stride, b.width, (uint32_t)tf.size(), 0, 0, miss};
        uint32_t maxb = 0;
        auto flush_lpf = [&]() {
            if (cur.n_feat == 0) return;
            cur.local_bins = maxb * 32;
            // 16-byte chunks of the record holding the tile's bins (staged kernel)
            uint32_t lo = ~0u, hi = 0;
            for (uint32_t i = cur.feat_begin; i < cur.feat_begin + cur.n_feat; i++) {
                lo = std::min(lo, tf[i].byte_off);
                hi = std::max(hi, tf[i].byte_off + b.width);
            }
            cur.chunk0 = lo / 16;
            cur.n_chunks = (hi + 15) / 16 - cur.chunk0;
            max_chunks = std::max(max_chunks, cur.n_chunks);
            lpf[wi].push_back(cur);
            smem_lpf = std::max(smem_lpf, (size_t)cur.local_bins * 16);
            cur.feat_begin = (uint32_t)tf.size();
            cur.n_feat = 0;
            maxb = 0;
        };
        for (uint32_t f : b.feats) {
            if (!en[f] || nbins_[f] > kLpfMaxBins) continue;
            if (cur.n_feat == 32) flush_lpf();
            tf.push_back(TileFeat{feat_byte_[f], 0, nbins_[f], gbin(f)});
            maxb = std::max(maxb, nbins_[f]);
            cur.n_feat++;
        }
        flush_lpf();
        // wide tiles
        TileDesc wd{b.base, b.stride, b.width, (uint32_t)tf.size(), 0, 0, miss};
        uint32_t wlo = ~0u, whi = 0;
        maxb = 0;
        auto flush_wide = [&]() {
            if (wd.n_feat == 0) return;
            wd.local_bins = maxb * kWideLanes;
            wd.chunk0 = wlo / 16;
            wd.n_chunks = (whi + 15) / 16 - wd.chunk0;
            max_chunks_wide = std::max(max_chunks_wide, wd.n_chunks);
            wide.push_back(wd);
            smem_wide = std::max(smem_wide, hist_wide_bytes(maxb));
            wd.feat_begin = (uint32_t)tf.size();
            wd.n_feat = 0;
            maxb = 0;
            wlo = ~0u;
            whi = 0;
        };
        for (uint32_t f : b.feats) {
            if (!en[f] || !is_wide(f, b.width)) continue;
            const uint32_t lo = std::min(wlo, feat_byte_[f]), hi = std::max(whi, feat_byte_[f] + 2);
            if (wd.n_feat == kWideLanes || (hi + 15) / 16 - lo / 16 > kWideMaxChunks) flush_wide();
            wlo = std::min(wlo, feat_byte_[f]);
            whi = std::max(whi, feat_byte_[f] + 2);
            tf.push_back(TileFeat{feat_byte_[f], 0, nbins_[f], gbin(f)});
            maxb = std::max(maxb, nbins_[f]);
            wd.n_feat++;
        }
        flush_wide();
        // row-per-thread tiles for the rest
        TileDesc g{b.base, b.stride, b.width, (uint32_t)tf.size(), 0, 0, miss};
        auto flush_gen = [&]() {
            if (g.n_feat == 0) return;
            gen[wi].push_back(g);
            smem_gen = std::max(smem_gen, (size_t)g.local_bins * 16 + (size_t)g.n_feat * sizeof(TileFeat));
            g.feat_begin = (uint32_t)tf.size();
            g.n_feat = 0;
            g.local_bins = 0;
        };
        for (uint32_t f : b.feats) {
            if (!en[f] || nbins_[f] <= kLpfMaxBins || nbins_[f] > max_local || is_wide(f, b.width)) continue;
            if (g.n_feat == 64 || g.local_bins + nbins_[f] > max_local) flush_gen();
            tf.push_back(TileFeat{feat_byte_[f], g.local_bins, nbins_[f], gbin(f)});
            g.local_bins += nbins_[f];
            g.n_feat++;
        }
        flush_gen();
        // features with more bins than the shared-memory budget (categorical
        // features of many codes): tiles without a shared histogram, updates
        // added to the node histogram directly
        TileDesc dt{b.base, b.stride, b.width, (uint32_t)tf.size(), 0, 0, miss};
        for (uint32_t f : b.feats) {
            if (!en[f] || nbins_[f] <= max_local || is_wide(f, b.width)) continue;
            if (dt.n_feat == 64) {
                direct[wi].push_back(dt);
                dt.feat_begin = (uint32_t)tf.size();
                dt.n_feat = 0;
            }
            tf.push_back(TileFeat{feat_byte_[f], 0, nbins_[f], gbin(f)});
            dt.n_feat++;
        }
        if (dt.n_feat) direct[wi].push_back(dt);
    }
    for (int w = 0; w < 2; w++)
        for (const TileDesc& t : direct[w]) smem_gen = std::max(smem_gen, (size_t)t.n_feat * sizeof(TileFeat));
    std::vector<TileDesc> all;
    // mean bins per tile of each launch (the fixed clear-and-flush work of a CTA)
    auto mean_bins = [&](const std::vector<TileDesc>& v) -> uint64_t {
        uint64_t b = 0;
        for (const TileDesc& t : v)
            for (uint32_t i = 0; i < t.n_feat; i++) b += tf[t.feat_begin + i].nbins;
        return v.empty() ? 0 : b / v.size();
    };
    for (int w = 0; w < 2; w++) {
        tile_bins_gen_[w] = mean_bins(gen[w]);
        tile_bins_lpf_[w] = mean_bins(lpf[w]);
        tile_bins_direct_[w] = mean_bins(direct[w]);
    }
    tile_bins_wide_ = mean_bins(wide);
    for (int w = 0; w < 2; w++) { tile_off_gen_[w] = (uint32_t)all.size(); n_gen_[w] = (uint32_t)gen[w].size(); all.insert(all.end(), gen[w].begin(), gen[w].end()); }
    for (int w = 0; w < 2; w++) { tile_off_lpf_[w] = (uint32_t)all.size(); n_lpf_[w] = (uint32_t)lpf[w].size(); all.insert(all.end(), lpf[w].begin(), lpf[w].end()); }
    tile_off_wide_ = (uint32_t)all.size();
    n_wide_ = (uint32_t)wide.size();
    all.insert(all.end(), wide.begin(), wide.end());
    for (int w = 0; w < 2; w++) { tile_off_direct_[w] = (uint32_t)all.size(); n_direct_[w] = (uint32_t)direct[w].size(); all.insert(all.end(), direct[w].begin(), direct[w].end()); }
    d_tiles_.alloc(sizeof(TileDesc) * std::max<size_t>(all.size(), 1));
    d_tfeat_.alloc(sizeof(TileFeat) * std::max<size_t>(tf.size(), 1));
    if (!all.empty())
        FB_CUDA_CHECK(cudaMemcpyAsync(d_tiles_.p, all.data(), sizeof(TileDesc) * all.size(), cudaMemcpyHostToDevice, s_));
    if (!tf.empty())
        FB_CUDA_CHECK(cudaMemcpyAsync(d_tfeat_.p, tf.data(), sizeof(TileFeat) * tf.size(), cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_enabled_.p, en.data(), F_, cudaMemcpyHostToDevice, s_));
    tile_smem_ = smem_gen;
    tile_smem_lpf_ = smem_lpf;
    set_hist_smem_limit((int)tile_smem_);
    set_hist_lpf_smem_limit((int)tile_smem_lpf_);
    // staged lane-per-feature kernel: 4 stages when the histogram leaves room
    // for them in the 227 KiB a CTA may use, else 2, else the unstaged kernel
    const size_t kMaxSmem = 227 * 1024;
    hist_stages_ = 0;
    tile_smem_stage_ = 0;
    if (max_chunks > 0) {
        for (int st : {4, 2}) {
            // + one discard row of 4 planes x 32 lanes
            const size_t need = smem_lpf + 512 + hist_stage_bytes(max_chunks, st);
            if (need <= kMaxSmem) {
                hist_stages_ = st;
                tile_smem_stage_ = need;
                break;
            }
        }
        if (hist_stages_) set_hist_stage_smem_limit((int)tile_smem_stage_);
    }
    // wide tiles: at most 4 chunks a record, so 4 stages always fit
    // (128.5 KiB + 32 warps x 4 x 8 rows x 80 B)
    wide_stages_ = 4;
    tile_smem_wide_ = smem_wide + hist_stage_bytes(std::max(max_chunks_wide, 1u), wide_stages_);
    if (n_wide_) set_hist_wide_smem_limit((int)tile_smem_wide_);
    sync();
    last_enabled_ = en;
    tiles_rank_major_ = rank_major;
    tiles_valid_ = true;
}

// One histogram pass over the accumulate rows of the current level (all tiles).
void TrainCtx::launch_histograms(const uint32_t* rows, const NodeInfo* nodes, const uint32_t* acc_list,
                                 const unsigned long long* acc_prefix, uint64_t rows_upper, Pair* out,
                                 unsigned long long slot) {
    const TileDesc* T = d_tiles_.as<TileDesc>();
    const TileFeat* TF = d_tfeat_.as<TileFeat>();
    if (!out) out = hist_acc_.as<Pair>();
    if (!slot) slot = std::max<uint64_t>(total_bins_, 1);
    // CTAs per feature tile.  Each CTA clears and flushes (global atomics
    // into the same node bins as its tile's other CTAs) a shared histogram of
    // its tile's bins whatever its row count, so a CTA should get rows in
    // proportion to its tile's bins: with many tiles and few rows (C2: 38
    // tiles of 32 features, 400k rows) a full grid per tile made that fixed
    // work dominate (5624 CTAs of ~2700 rows, 0.85 ms per level).  The
    // launch still fills every SM once (the kernels are issue-bound: idle SMs
    // cost more than extra flushes), and beyond one wave its CTAs are
    // snapped to whole waves (a nearly empty last wave costs a full one).
    // Rows per CTA per tile bin, measured on B200 (s / 100 rounds at factors
    // 1 / 4 / 16): lane-per-feature tiles 4 (C2: 0.703 / 0.589 / 0.631), wide
    // tiles 16 (C3: 1.003 / 1.002 / 0.844); C1 and C0 fill one wave at any.
    auto per_tile = [&](uint32_t slots, uint32_t n_tiles, uint64_t tile_bins, uint64_t min_rows,
                        uint64_t rows_per_bin) {
        if (n_tiles == 0) return 1u;
        const uint64_t want_rows = std::max<uint64_t>(min_rows, rows_per_bin * tile_bins);
        const uint64_t by_rows = std::max<uint64_t>(1, ceil_div(rows_upper, std::max<uint64_t>(want_rows, 1)));
        const uint64_t fill = std::min<uint64_t>(std::max<uint32_t>(1, slots / n_tiles),
                                                 std::max<uint64_t>(1, ceil_div(rows_upper, min_rows)));
        uint64_t g = std::min<uint64_t>(std::max(by_rows, fill), slots);
        const uint64_t total = g * n_tiles;
        if (total > slots) {
            const uint64_t waves = std::max<uint64_t>(1, (total + slots / 2) / slots);
            g = std::max<uint64_t>(1, waves * slots / n_tiles);
        }
        return (uint32_t)g;
    };
    const size_t lpf_smem = hist_stages_ ? tile_smem_stage_ : tile_smem_lpf_;
    const int per_sm = lpf_smem + 1024 <= 113 * 1024 ? 2 : 1;
    for (int w = 0; w < 2; w++) {
        const uint32_t grid_gen = per_tile(148 * 2, n_gen_[w], tile_bins_gen_[w], 1024, 4);
        const uint32_t grid_lpf = per_tile(148u * per_sm, n_lpf_[w], tile_bins_lpf_[w], 512, 4);
        launch_hist(w + 1, T + tile_off_gen_[w], n_gen_[w], TF, rows, fixed_.as<Pair>(), nodes, acc_list, acc_prefix,
                    state_.as<TreeState>(), out, slot, grid_gen, tile_smem_, s_);
        if (hist_stages_)
            launch_hist_stage(w + 1, hist_stages_, T + tile_off_lpf_[w], n_lpf_[w], TF, rows, fixed_.as<Pair>(), nodes,
                              acc_list, acc_prefix, state_.as<TreeState>(), out, slot, grid_lpf,
                              lpf_smem, s_);
        else
            launch_hist_lpf(w + 1, T + tile_off_lpf_[w], n_lpf_[w], TF, rows, fixed_.as<Pair>(), nodes, acc_list,
                            acc_prefix, state_.as<TreeState>(), out, slot, grid_lpf, tile_smem_lpf_,
                            s_);
    }
    for (int w = 0; w < 2; w++)
        if (n_direct_[w])
            launch_hist(w + 1, T + tile_off_direct_[w], n_direct_[w], TF, rows, fixed_.as<Pair>(), nodes, acc_list,
                        acc_prefix, state_.as<TreeState>(), out, slot,
                        per_tile(148 * 2, n_direct_[w], tile_bins_direct_[w], 1024, 4),
                        tile_smem_, s_);
    if (n_wide_) {
        const uint32_t grid_wide = per_tile(148u, n_wide_, tile_bins_wide_, 512, 16);
        launch_hist_wide(wide_stages_, T + tile_off_wide_, n_wide_, TF, rows, fixed_.as<Pair>(), nodes, acc_list,
                         acc_prefix, state_.as<TreeState>(), out, slot, grid_wide, tile_smem_wide_,
                         s_);
    }
}

// The split search's feature lists for [a.feat_lo, a.feat_hi): numeric
// features of up to 256 bins (a warp each) and the rest (a CTA each).
void TrainCtx::set_split_lists(LevelArgs& a) {
    if (split_lists_lo_ != a.feat_lo || split_lists_hi_ != a.feat_hi || !d_split_lists_.p) {
        std::vector<uint32_t> num, cta;
        for (uint32_t f = a.feat_lo; f < a.feat_hi; f++)
            ((nbins_[f] <= 256 && !cat_[f]) ? num : cta).push_back(f);
        n_split_num_ = (uint32_t)num.size();
        n_split_cta_ = (uint32_t)cta.size();
        split_lists_host_ = num;
        split_lists_host_.insert(split_lists_host_.end(), cta.begin(), cta.end());
        d_split_lists_.alloc(4 * std::max<size_t>(split_lists_host_.size(), 1));
        if (!split_lists_host_.empty())
            FB_CUDA_CHECK(cudaMemcpyAsync(d_split_lists_.p, split_lists_host_.data(), 4 * split_lists_host_.size(),
                                          cudaMemcpyHostToDevice, s_));
        split_lists_lo_ = a.feat_lo;
        split_lists_hi_ = a.feat_hi;
    }
    a.split_num = d_split_lists_.as<uint32_t>();
    a.n_split_num = n_split_num_;
    a.split_cta = d_split_lists_.as<uint32_t>() + n_split_num_;
    a.n_split_cta = n_split_cta_;
}

LevelArgs TrainCtx::level_args(const fbgpu_tree_params& tp) const {
    LevelArgs a{};
    a.n_features = F_;
    a.max_leaves = tp.max_leaves;
    a.sp = ScoreParams{tp.lambda, tp.gamma, tp.min_child_weight, tp.alpha, tp.max_delta_step, tp.eta, 1.0, 1.0};
    a.scales = reinterpret_cast<const double*>(sums_.as<unsigned long long>() + 4);
    a.hoff = d_hoff_.as<uint32_t>();
    a.enabled = d_enabled_.as<uint8_t>();
    a.mono = tp.monotone ? d_mono_.as<int8_t>() : nullptr;
    a.is_cat = has_cat_ ? d_cat_.as<uint8_t>() : nullptr;
    a.max_onehot = tp.max_cat_to_onehot;
    a.max_cat_threshold = tp.max_cat_threshold;
    a.floc = d_floc_.as<FeatLoc>();
    a.floc_rec = d_floc_rec_.as<FeatLoc>();
    a.st = state_.as<TreeState>();
    a.hist_acc = hist_acc_.as<Pair>();
    a.slot_pairs = std::max<uint64_t>(total_bins_, 1);
    a.feat_lo = 0;
    a.feat_hi = F_;
    a.bin_lo = 0;
    a.feat_best = feat_best_.as<SplitRec>();
    a.cat_words = cat_words_;
    a.cat_slot = d_cat_slot_.as<uint32_t>();
    a.n_cat = n_cat_;
    a.feat_cats = feat_cats_.as<uint32_t>();
    a.node_best = node_best_.as<SplitRec>();
    a.node_cats = node_cats_.as<uint32_t>();
    a.split = split_.as<SplitDesc>();
    a.chunk_left = chunk_left_.as<uint32_t>();
    a.chunk_off = chunk_off_.as<uint32_t>();
    a.dirflags = dirflags_.as<uint8_t>();
    a.node_left = node_left_.as<uint32_t>();
    // sharded: the accumulated child is chosen by global hessian sums, so no
    // per-level count allreduce is needed (the choice never changes the model)
    a.node_left_global = comm_ ? nullptr : node_left_.as<uint32_t>();
    a.pred = pred_.as<float>() + (size_t)pred_col_ * n_;
    a.trec = trec_.as<TreeRec>();
    a.tcats = tcats_.as<uint32_t>();
    return a;
}

// Contiguous feature ranges, one per rank, with about total_bins / N bins
// each: rank r scores the features from the first one whose bins start at or
// after r / N of all bins.  chunk_pairs_ is the largest range's bin count.
void TrainCtx::setup_split_shards() {
    const uint32_t N = (uint32_t)nranks_;
    if (total_bins_ >= (1u << 24)) throw InputError("the feature-sharded split search packs bin offsets in 24 bits");
    rank_feat_lo_.assign(N + 1, F_);
    rank_bin_lo_.assign(N + 1, (uint32_t)total_bins_);
    uint32_t f = 0;
    for (uint32_t r = 0; r < N; r++) {
        const uint64_t target = total_bins_ * r / N;
        while (f < F_ && hoff_[f] < target) f++;
        rank_feat_lo_[r] = f;
        rank_bin_lo_[r] = hoff_[f];
    }
    feat_rank_.assign(F_, 0);
    chunk_pairs_ = 1;
    for (uint32_t r = 0; r < N; r++) {
        for (uint32_t g = rank_feat_lo_[r]; g < rank_feat_lo_[r + 1]; g++) feat_rank_[g] = r;
        chunk_pairs_ = std::max<uint64_t>(chunk_pairs_, rank_bin_lo_[r + 1] - rank_bin_lo_[r]);
    }
    split_shard_ = true;
}

// Lossguide grows the same tree as depthwise growth when max_leaves cannot
// bind (0, or at least 2^max_depth leaves): every leaf with a split is popped
// before the budget runs out (lossguide.rs:555-700), so only the node order
// differs.
bool lossguide_is_levelwise(const fbgpu_tree_params& tp) {
    return tp.max_leaves == 0 || tp.max_depth >= 31 || tp.max_leaves >= (1u << tp.max_depth);
}

// Best-first pop order over a grown tree (lossguide.rs:46-53 ordering: larger
// gain by f32 total order first, then the lower node id; children get ids
// in pop order, left then right).
void lossguide_order(const TreeRec* rec, uint32_t nn, std::vector<uint32_t>& old_of_new,
                     std::vector<uint32_t>& new_of_old) {
    struct E {
        int32_t key;   // f32 gain as a total-order integer
        uint32_t id;   // new id
        uint32_t old;  // depthwise id
    };
    auto total_key = [](float g) {
        int32_t i;
        std::memcpy(&i, &g, 4);
        return i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
    };
    auto less = [](const E& a, const E& b) { return a.key != b.key ? a.key < b.key : a.id > b.id; };
    old_of_new.assign(nn, 0);
    new_of_old.assign(nn, 0);
    uint32_t next = 1;
    std::vector<E> heap;
    if (!(rec[0].flags & 1u)) heap.push_back({total_key(rec[0].gain), 0, 0});
    while (!heap.empty()) {
        std::pop_heap(heap.begin(), heap.end(), less);
        const E e = heap.back();
        heap.pop_back();
        const int32_t kids[2] = {rec[e.old].left, rec[e.old].right};
        for (int32_t c : kids) {
            if (c < 0 || (uint32_t)c >= nn || next >= nn) throw std::runtime_error("device tree is malformed");
            new_of_old[c] = next;
            old_of_new[next] = (uint32_t)c;
            if (!(rec[c].flags & 1u)) {
                heap.push_back({total_key(rec[c].gain), next, (uint32_t)c});
                std::push_heap(heap.begin(), heap.end(), less);
            }
            next++;
        }
    }
    if (next != nn) throw std::runtime_error("device tree is malformed");
}

void TrainCtx::launch_graph(cudaGraph_t g, int slot, int segment) {
    if (segment >= kTreeSegments) throw std::runtime_error("more graph segments than a tree has levels");
    cudaGraphExec_t& e = tree_exec_[slot][segment];
    if (e) {
        cudaGraphExecUpdateResultInfo info{};
        if (cudaGraphExecUpdate(e, g, &info) != cudaSuccess) {  // another shape: instantiate anew
            (void)cudaGetLastError();
            cudaGraphExecDestroy(e);
            e = nullptr;
        }
    }
    const cudaError_t inst = e ? cudaSuccess : cudaGraphInstantiate(&e, g, 0);
    cudaGraphDestroy(g);
    FB_CUDA_CHECK(inst);
    FB_CUDA_CHECK(cudaGraphLaunch(e, s_));
}

bool TrainCtx::tree_async(const fbgpu_tree_params& tp) const {
    return tp.grow_policy == 0 || lossguide_is_levelwise(tp);
}

void TrainCtx::wait_event(cudaEvent_t ev) {
    if (comm_) comm_->wait_event(ev);
    else FB_CUDA_CHECK(cudaEventSynchronize(ev));
}

void TrainCtx::build_tree(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* out) {
    if (!tree_async(tp)) {
        build_tree_launch(tp, enabled, out);  // best-first: grown and read back here
        return;
    }
    if (slots_pending_) throw InputError("collect the launched trees before building one synchronously");
    build_tree_launch(tp, enabled, nullptr);
    build_tree_collect(out);
}

void TrainCtx::build_tree_launch(const fbgpu_tree_params& tp, const uint8_t* enabled) {
    if (!tree_async(tp)) throw InputError("this tree needs the host while it grows (best-first lossguide)");
    build_tree_launch(tp, enabled, nullptr);
}

void TrainCtx::build_tree_launch(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* lg_out) {
    const NextGrad ng = next_grad_;
    next_grad_.set = false;
    fused_grad_.set = false;
    ensure_features();
    if (tp.max_depth > 14) throw InputError("max_depth must be in 0..=14");
    const bool lossguide = tp.grow_policy != 0;
    if (n_ == 0) throw InputError("training data must have at least one row");
    const bool best_first = lossguide && !lossguide_is_levelwise(tp);
    ensure_tree_buffers(tp.max_depth, tp.max_leaves, best_first);
    // Row-sharded depthwise trees with large level histograms score splits
    // per rank on its own features: a reduce-scatter of the level's
    // histograms (half the bytes of an all-reduce) and a gather of the
    // per-node winners (one more collective and a merge kernel per level).
    // FBGPU_SPLIT_SHARD=1 / 0 forces either form.
    static const int split_shard_env = [] {
        const char* e = std::getenv("FBGPU_SPLIT_SHARD");
        return e ? (std::string(e) == "0" ? 0 : 1) : -1;
    }();
    const bool wide_levels = 16ull * max_acc_ * total_bins_ >= (32ull << 20);
    const bool rs_mode = comm_ && nranks_ > 1 && !best_first &&
                         (split_shard_env >= 0 ? split_shard_env == 1 : wide_levels);
    if (rs_mode) {
        if (!split_shard_) setup_split_shards();
        const uint64_t lvl = max_level_nodes_;
        const uint64_t block = (uint64_t)max_acc_ * chunk_pairs_;
        if (hist_acc_.bytes < 16ull * nranks_ * block + 16) hist_acc_.alloc(16ull * nranks_ * block + 16);
        if (hist_rs_.bytes < 16ull * block) hist_rs_.alloc(16ull * block);
        if (best_all_.bytes < sizeof(SplitRec) * nranks_ * lvl) best_all_.alloc(sizeof(SplitRec) * nranks_ * lvl);
        if (cats_all_.bytes < 4ull * cat_words_ * nranks_ * lvl) cats_all_.alloc(4ull * cat_words_ * nranks_ * lvl);
        h_stride_.reserve(8 * 16);
    }
    plan_tiles(enabled, rs_mode);
    if (tp.monotone) {
        std::vector<int8_t> m(tp.monotone, tp.monotone + F_);
        if (m != last_mono_) {
            FB_CUDA_CHECK(cudaMemcpyAsync(d_mono_.p, m.data(), F_, cudaMemcpyHostToDevice, s_));
            last_mono_ = m;
        }
    }
    if (best_first) {
        if (slots_pending_) throw InputError("collect the launched trees before growing a best-first tree");
        ensure_lossguide_buffers(tp.max_leaves);
        build_tree_lossguide(tp, enabled, lg_out);
        return;
    }
    if (slots_pending_ == 2) throw InputError("two trees are in flight: collect one before launching another");
    ReadSlot& S = slot_[slot_next_];
    LevelArgs a = level_args(tp);
    // the one-CTA level steps ride in the last CTA of the kernel before them
    if (!fuse_.p) {
        fuse_.alloc(16);
        FB_CUDA_CHECK(cudaMemsetAsync(fuse_.p, 0, 16, s_));
    }
    a.fuse = fuse_.as<unsigned int>();
    a.part_cnt = part_cnt_.as<unsigned long long>();
    // Leaf values reach the margins either by one walk of the finished tree
    // per row (k_tree_walk; the last level then needs no partition) or per
    // partition chunk (k_part_level for nodes that stop early, k_part_final
    // for the last level).  The walk streams every row's record once and
    // updates the margins in row order; the partition path updates them in
    // arena order, one scattered sector per row.  Measured on B200: the walk
    // is faster up to a few million local rows, and beyond when its fast form
    // applies (the tree in shared memory, every feature in one staged record
    // block): C1, 11M rows, 0.265 against 0.273 s / 100 rounds.
    // FBGPU_WALK=0 / 1 forces one.
    static const int walk_env = [] {
        const char* e = std::getenv("FBGPU_WALK");
        return e ? std::atoi(e) : -1;
    }();
    if (blocks_.size() == 1 && blocks_[0]->stride <= 64 && blocks_[0]->stride % 4 == 0) {
        a.walk_rec = blocks_[0]->base;
        a.walk_stride = blocks_[0]->stride;
    }
    uint64_t max_nodes = (2ull << tp.max_depth) - 1;  // max_depth <= 14
    if (tp.max_leaves) max_nodes = std::min<uint64_t>(max_nodes, 2ull * tp.max_leaves - 1);
    const bool walk_fast = a.walk_rec != nullptr && max_nodes <= kWalkNodes;
    a.walk = walk_env >= 0 ? (walk_env ? 1u : 0u) : ((n_ <= (4ull << 20) || walk_fast) ? 1u : 0u);
    const uint32_t maxd = tp.max_depth;
    const uint32_t W = cat_words_;
    if (rs_mode) {
        // the split reads this rank's block of the reduce-scattered histograms,
        // its node slots hold this rank's bins only
        a.hist_acc = hist_rs_.as<Pair>();
        a.slot_pairs = chunk_pairs_;
        a.feat_lo = rank_feat_lo_[rank_];
        a.feat_hi = rank_feat_lo_[rank_ + 1];
        a.bin_lo = rank_bin_lo_[rank_];
    }
    // host-side set-up first: from here to the readback nothing allocates,
    // uploads from pageable memory or waits, so that span can be captured
    set_split_lists(a);
    S.tree.reserve(sizeof(TreeRec) * max_tree_nodes_ + 4ull * W * max_tree_nodes_ + sizeof(TreeState));
    S.small.reserve(16 * 16 + 8);
    // Without per-level statistics the tree's launches (about 40) are
    // captured into CUDA graphs and launched as one graph per segment, so the
    // device runs them back to back: one segment per tree on one GPU.  The
    // graphs are captured again every tree and the slot's executable graphs
    // updated from them (cudaGraphExecUpdate), so they never replay stale
    // arguments; the capture costs host time that the pipelined rounds
    // overlap with the device's.  FBGPU_GRAPHS=0 launches the kernels one by
    // one.
    static const bool graphs_env = [] {
        const char* e = std::getenv("FBGPU_GRAPHS");
        return !(e && std::string(e) == "0");
    }();
    // the events and the readback copies stay outside the graph: the host
    // waits on them, and an event recorded during a capture is a graph
    // dependency, not one the host can wait for
    FB_CUDA_CHECK(cudaEventRecord(S.ev0, s_));
    // Sharded: the collectives stay outside the graphs.  Each span of kernels
    // between two of them (the level's split, partition and the next level's
    // histograms) is captured and launched as one segment.  The
    // feature-sharded form and a root-only tree keep launching kernel by kernel.
    const bool graphs = graphs_env && !stats_ && !rs_mode && !(comm_ && root_pending_ && maxd == 0);
    CaptureGuard capture(s_, graphs);
    int segment = 0;
    int cur = 0;
    launch_iota(rows_[0].as<uint32_t>(), (uint32_t)n_, s_);
    a.nodes = nodes_[0].as<NodeInfo>();
    a.acc_list = acc_list_[0].as<uint32_t>();
    a.acc_prefix = acc_prefix_[0].as<unsigned long long>();
    a.chunk_prefix = chunk_prefix_[0].as<uint32_t>();
    a.rows_cur = rows_[0].as<uint32_t>();
    if (root_pending_ && (maxd == 0 || rs_mode)) reduce_root_sum(true);
    launch_tree_init(a, (uint32_t)n_, (uint32_t)cfg_.n_rows_global, sums_.as<unsigned long long>(), s_);
    for (uint32_t d = 0; d < maxd; d++) {
        const uint32_t max_m = (uint32_t)std::min<uint64_t>(1ull << d, max_level_nodes_);
        const uint32_t max_acc = d == 0 ? 1u : (uint32_t)std::min<uint64_t>(1ull << (d - 1), max_acc_);
        a.depth = d;
        a.last_level = d + 1 == maxd;
        a.nodes = nodes_[cur].as<NodeInfo>();
        a.next_nodes = nodes_[1 - cur].as<NodeInfo>();
        a.acc_list = acc_list_[cur].as<uint32_t>();
        a.acc_prefix = acc_prefix_[cur].as<unsigned long long>();
        a.next_acc_list = acc_list_[1 - cur].as<uint32_t>();
        a.next_acc_prefix = acc_prefix_[1 - cur].as<unsigned long long>();
        a.chunk_prefix = chunk_prefix_[cur].as<uint32_t>();
        a.next_chunk_prefix = chunk_prefix_[1 - cur].as<uint32_t>();
        a.hist_cur = hist_[d & 1].as<Pair>();
        a.hist_prev = hist_[(d + 1) & 1].as<Pair>();
        a.rows_cur = rows_[cur].as<uint32_t>();
        a.rows_next = rows_[1 - cur].as<uint32_t>();
        const uint64_t block = (uint64_t)max_acc * chunk_pairs_;  // rs_mode: pairs of one rank's block
        // the level's accumulate histograms start at zero: the root level's
        // here, the others zeroed by the previous level's k_part_level
        auto acc_bytes = [&](uint64_t acc) {
            return rs_mode ? 16ull * nranks_ * acc * chunk_pairs_ : 16ull * a.slot_pairs * acc;
        };
        if (d == 0) FB_CUDA_CHECK(cudaMemsetAsync(hist_acc_.p, 0, acc_bytes(max_acc), s_));
        if (stats_ && d < 15) {
            // this level's accumulate nodes and rows: TreeState bytes [8, 24) hold
            // leaf_count, acc_count (u32 each) and acc_total (u64)
            static_assert(offsetof(TreeState, acc_count) == 12 && offsetof(TreeState, acc_total) == 16,
                          "TreeState layout");
            FB_CUDA_CHECK(cudaMemcpyAsync(level_stats_.as<uint8_t>() + 16 * d,
                                          reinterpret_cast<uint8_t*>(state_.p) + 8, 16, cudaMemcpyDeviceToDevice, s_));
            FB_CUDA_CHECK(cudaEventRecord(S.hev[2 * d], s_));
        }
        const bool root_rides = d == 0 && root_pending_;
        if (root_rides)
            FB_CUDA_CHECK(cudaMemcpyAsync(hist_acc_.as<unsigned long long>() + 2ull * a.slot_pairs, sums_.p, 16,
                                          cudaMemcpyDeviceToDevice, s_));
        if (rs_mode) {
            // rank-major accumulate histograms ([rank][slot][rank's bins]); each
            // rank receives the sums of its own block
            uint64_t* hs = h_stride_.as<uint64_t>() + (d & 15);
            *hs = block;
            FB_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(state_.p) + offsetof(TreeState, rank_stride), hs,
                                          8, cudaMemcpyHostToDevice, s_));
            launch_histograms(a.rows_cur, a.nodes, a.acc_list, a.acc_prefix, n_, hist_acc_.as<Pair>(), chunk_pairs_);
            if (stats_ && d < 15) FB_CUDA_CHECK(cudaEventRecord(S.hevc[d], s_));
            comm_->reduce_scatter_u64(hist_acc_.p, hist_rs_.p, 2 * block, s_);
        } else {
            launch_histograms(a.rows_cur, a.nodes, a.acc_list, a.acc_prefix, n_);
            if (stats_ && comm_ && d < 15) FB_CUDA_CHECK(cudaEventRecord(S.hevc[d], s_));
            if (comm_ && capture.on) launch_graph(capture.end(), slot_next_, segment++);
            allreduce_u64(hist_acc_.p, 2ull * a.slot_pairs * max_acc + (root_rides ? 2 : 0), false);
            if (comm_ && graphs) capture.begin();
        }
        if (root_rides) {
            FB_CUDA_CHECK(cudaMemcpyAsync(sums_.p, hist_acc_.as<unsigned long long>() + 2ull * a.slot_pairs, 16,
                                          cudaMemcpyDeviceToDevice, s_));
            // the root again, now with the global sum (same spans and state)
            launch_tree_init(a, (uint32_t)n_, (uint32_t)cfg_.n_rows_global, sums_.as<unsigned long long>(), s_);
            root_pending_ = false;
        }
        if (stats_ && d < 15) FB_CUDA_CHECK(cudaEventRecord(S.hev[2 * d + 1], s_));
        const uint32_t max_chunks = ceil_div(std::max<uint64_t>(n_, 1), kChunkRows) + max_m;
        if (rs_mode) {
            // this rank's best split per node over its features, every rank's
            // winners gathered, merged and decided
            launch_split(a, max_m, s_);
            comm_->all_gather_bytes(node_best_.p, best_all_.p, sizeof(SplitRec) * max_m, s_);
            if (has_cat_) comm_->all_gather_bytes(node_cats_.p, cats_all_.p, 4ull * cat_words_ * max_m, s_);
            launch_merge_decide(a, best_all_.as<SplitRec>(), cats_all_.as<uint32_t>(), (uint32_t)nranks_, max_m, s_);
        } else {
            launch_split_decide(a, max_m, s_);
        }
        // the last level's children are final leaves: with the walk they need
        // nothing here, otherwise their leaf values go to the margins now
        if (!a.last_level) {
            const uint64_t next_acc = std::min<uint64_t>(1ull << d, max_acc_);
            a.hist_zero = hist_acc_.as<unsigned long long>();
            a.hist_zero_words = acc_bytes(next_acc) / 8;
            launch_part_level(a, max_chunks, s_);
            a.hist_zero = nullptr;
            a.hist_zero_words = 0;
        }
        else if (!a.walk) launch_part_final(a, max_chunks, s_);
        cur = 1 - cur;
    }
    a.nodes = nodes_[cur].as<NodeInfo>();
    a.chunk_prefix = chunk_prefix_[cur].as<uint32_t>();
    a.rows_cur = rows_[cur].as<uint32_t>();
    const uint32_t last_m = (uint32_t)std::min<uint64_t>(1ull << maxd, max_level_nodes_);
    if (a.walk && ng.set) {
        // the next round's gradients from the new margins, in the walk; its
        // bounds start from zero (this round's were read by its scales)
        FB_CUDA_CHECK(cudaMemsetAsync(sums_.as<unsigned long long>() + 2, 0, 16, s_));
        GradArgs ga = grad_args();
        ga.sub_th = ng.th; ga.sub_seed = ng.seed; ga.sub_tree = ng.tree;
        ga.objective = ng.objective;
        launch_tree_walk(a, (uint32_t)n_, s_, &ga, ng.fast ? 1 : (ng.objective == 1 ? 2 : 0));
        fused_grad_ = ng;
    } else if (a.walk)
        launch_tree_walk(a, (uint32_t)n_, s_);
    else if (maxd == 0)  // the root is the only leaf
        launch_leaf_final(a, ceil_div(std::max<uint64_t>(n_, 1), kChunkRows) + last_m, s_);
    FB_CUDA_CHECK(cudaGetLastError());
    if (capture.on) launch_graph(capture.end(), slot_next_, segment);
    FB_CUDA_CHECK(cudaEventRecord(S.ev1, s_));
    // the result into this slot's pinned buffers, in stream order (the next
    // tree's kernels overwrite the device copies only after these)
    TreeRec* hrec = S.tree.as<TreeRec>();
    uint32_t* hcats = reinterpret_cast<uint32_t*>(hrec + max_tree_nodes_);
    TreeState* hst = reinterpret_cast<TreeState*>(hcats + (size_t)W * max_tree_nodes_);
    FB_CUDA_CHECK(cudaMemcpyAsync(hst, state_.p, sizeof(TreeState), cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(hrec, trec_.p, sizeof(TreeRec) * max_tree_nodes_, cudaMemcpyDeviceToHost, s_));
    if (has_cat_)
        FB_CUDA_CHECK(cudaMemcpyAsync(hcats, tcats_.p, 4ull * W * max_tree_nodes_, cudaMemcpyDeviceToHost, s_));
    uint64_t* lvl = S.small.as<uint64_t>();  // 16 levels x 16 bytes
    if (stats_) FB_CUDA_CHECK(cudaMemcpyAsync(lvl, level_stats_.p, 16 * 16, cudaMemcpyDeviceToHost, s_));
    S.scale_err = scale_err_pending_;
    scale_err_pending_ = false;
    if (S.scale_err)
        FB_CUDA_CHECK(cudaMemcpyAsync(lvl + 32, sums_.as<unsigned long long>() + 6, 8, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaEventRecord(S.done, s_));
    S.lossguide = lossguide;
    S.max_nodes = max_tree_nodes_;
    S.stats = stats_;
    S.maxd = maxd;
    S.W = W;
    if (stats_) {
        S.row_bytes = S.bins = S.feats = 0;  // enabled features of this tree
        for (uint32_t f = 0; f < F_; f++)
            if (last_enabled_[f]) { S.row_bytes += width_[f]; S.bins += nbins_[f]; S.feats += 1; }
        S.launches_per_level = (n_gen_[0] ? 1 : 0) + (n_gen_[1] ? 1 : 0) + (n_lpf_[0] ? 1 : 0) + (n_lpf_[1] ? 1 : 0) +
                               (n_wide_ ? 1 : 0) + (n_direct_[0] ? 1 : 0) + (n_direct_[1] ? 1 : 0);
    }
    slot_next_ = 1 - slot_next_;
    slots_pending_++;
}

void TrainCtx::build_tree_collect(fbgpu_tree_out* out) {
    if (slots_pending_ == 0) throw InputError("no launched tree to collect");
    ReadSlot& S = slot_[(slot_next_ + 2 - slots_pending_) % 2];
    slots_pending_--;
    wait_event(S.done);
    const uint32_t W = S.W;
    const TreeRec* hrec = S.tree.as<TreeRec>();
    const uint32_t* hcats = reinterpret_cast<const uint32_t*>(hrec + S.max_nodes);
    const TreeState* hst = reinterpret_cast<const TreeState*>(hcats + (size_t)W * S.max_nodes);
    const uint64_t* lvl = S.small.as<uint64_t>();
    FB_CUDA_CHECK(cudaEventElapsedTime(&last_tree_ms_, S.ev0, S.ev1));
    if (S.scale_err && lvl[32]) throw InputError("non-finite gradient or Hessian");
    if (S.stats) {
        for (uint32_t d = 0; d < std::min<uint32_t>(S.maxd, 15); d++) {
            float ms = 0.0f;
            FB_CUDA_CHECK(cudaEventElapsedTime(&ms, S.hev[2 * d], S.hev[2 * d + 1]));
            if (comm_) {
                float cms = 0.0f;
                FB_CUDA_CHECK(cudaEventElapsedTime(&cms, S.hevc[d], S.hev[2 * d + 1]));
                comm_ms_ += cms;
            }
            const uint64_t acc_nodes = lvl[2 * d] >> 32, rows = lvl[2 * d + 1];
            hist_ms_ += ms;
            hist_launches_ += S.launches_per_level;
            hist_bytes_ += (double)rows * (S.row_bytes + 16 + (d ? 4 : 0)) + (double)acc_nodes * S.bins * 16.0;
            hist_updates_ += (double)rows * S.feats;
        }
    }
    const bool lossguide = S.lossguide;
    const uint32_t nn = hst->n_tree_nodes;
    if (nn == 0 || nn > S.max_nodes) throw std::runtime_error("device tree has an invalid node count");
    if (!out) return;
    if (out->capacity < nn) throw InputError("fbgpu_tree_out capacity is smaller than the tree");
    const uint32_t out_w = out->cat_words ? out->cat_words : 8u;
    if (out->cats && out_w < W)
        throw InputError("fbgpu_tree_out.cat_words is smaller than the context's category sets (fbgpu_ctx_cat_words)");
    out->n_nodes = nn;
    // lossguide: the same splits, numbered in best-first pop order
    std::vector<uint32_t> old_of_new, new_of_old;
    if (lossguide) lossguide_order(hrec, nn, old_of_new, new_of_old);
    for (uint32_t i = 0; i < nn; i++) {
        const uint32_t o = lossguide ? old_of_new[i] : i;
        const TreeRec& r = hrec[o];
        const uint32_t ci = o;  // categories stay with their node
        if (out->left) out->left[i] = r.left < 0 || !lossguide ? r.left : (int32_t)new_of_old[r.left];
        if (out->right) out->right[i] = r.right < 0 || !lossguide ? r.right : (int32_t)new_of_old[r.right];
        if (out->feat) out->feat[i] = r.feat;
        if (out->bin) out->bin[i] = r.bin;
        if (out->gain) out->gain[i] = r.gain;
        if (out->leaf) out->leaf[i] = r.leaf;
        if (out->hess) out->hess[i] = r.hess;
        if (out->flags) out->flags[i] = r.flags;
        if (out->cats) {
            for (uint32_t w = 0; w < out_w; w++)
                out->cats[(size_t)i * out_w + w] = (r.flags & 4u) && w < W ? hcats[(size_t)ci * W + w] : 0u;
        }
    }
}

void TrainCtx::download_margins(float* out) {
    FB_CUDA_CHECK(cudaMemcpyAsync(out, pred_.p, (size_t)K_ * n_ * 4, cudaMemcpyDeviceToHost, s_));
    sync();
}

// ---- component calls (kernel parity tests) --------------------------------
void TrainCtx::histogram(const uint32_t* rows, uint64_t n_sel, const int64_t* fixed, int64_t* out) {
    ensure_features();
    if (fixed) FB_CUDA_CHECK(cudaMemcpyAsync(fixed_.p, fixed, n_ * 16, cudaMemcpyHostToDevice, s_));
    ensure_tree_buffers(std::max<uint32_t>(buf_depth_ == 0xffffffffu ? 1 : buf_depth_, 1), buf_leaves_ == 0xffffffffu ? 0 : buf_leaves_);
    plan_tiles(nullptr);
    std::vector<uint32_t> all;
    if (!rows) {
        all.resize(n_);
        for (uint64_t i = 0; i < n_; i++) all[i] = (uint32_t)i;
        rows = all.data();
        n_sel = n_;
    }
    DevMem drows;
    drows.alloc(std::max<uint64_t>(n_sel, 1) * 4);
    FB_CUDA_CHECK(cudaMemcpyAsync(drows.p, rows, n_sel * 4, cudaMemcpyHostToDevice, s_));
    NodeInfo ni{};
    ni.start = 0; ni.len = (uint32_t)n_sel; ni.tree_id = 0; ni.parent_slot = -1; ni.acc_slot = 0;
    uint32_t acc_list = 0;
    unsigned long long acc_prefix[2] = {0, n_sel};
    TreeState st{};
    st.m = 1; st.acc_count = 1; st.acc_total = n_sel;
    FB_CUDA_CHECK(cudaMemcpyAsync(nodes_[0].p, &ni, sizeof ni, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(acc_list_[0].p, &acc_list, 4, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(acc_prefix_[0].p, acc_prefix, 16, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(state_.p, &st, sizeof st, cudaMemcpyHostToDevice, s_));
    const unsigned long long slot = std::max<uint64_t>(total_bins_, 1);
    FB_CUDA_CHECK(cudaMemsetAsync(hist_acc_.p, 0, 16 * slot, s_));
    launch_histograms(drows.as<uint32_t>(), nodes_[0].as<NodeInfo>(), acc_list_[0].as<uint32_t>(),
                      acc_prefix_[0].as<unsigned long long>(), n_sel);
    FB_CUDA_CHECK(cudaGetLastError());
    FB_CUDA_CHECK(cudaMemcpyAsync(out, hist_acc_.p, 16 * total_bins_, cudaMemcpyDeviceToHost, s_));
    sync();
}

void TrainCtx::eval_split(const int64_t* hist, const int64_t* node_sum, const double* scales,
                          const fbgpu_tree_params& tp, float lower, float upper, const uint8_t* enabled,
                          fbgpu_split* out) {
    ensure_features();
    ensure_tree_buffers(std::max<uint32_t>(buf_depth_, 1), buf_leaves_);
    std::vector<uint8_t> en(F_, 1);
    if (enabled) for (uint32_t f = 0; f < F_; f++) en[f] = enabled[f] ? 1 : 0;
    FB_CUDA_CHECK(cudaMemcpyAsync(d_enabled_.p, en.data(), F_, cudaMemcpyHostToDevice, s_));
    tiles_valid_ = false;
    if (tp.monotone) FB_CUDA_CHECK(cudaMemcpyAsync(d_mono_.p, tp.monotone, F_, cudaMemcpyHostToDevice, s_));
    last_mono_.clear();
    FB_CUDA_CHECK(cudaMemcpyAsync(hist_acc_.p, hist, 16 * total_bins_, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(sums_.as<unsigned long long>() + 4, scales, 16, cudaMemcpyHostToDevice, s_));
    NodeInfo ni{};
    ni.start = 0; ni.len = 0; ni.tree_id = 0; ni.parent_slot = -1; ni.acc_slot = 0;
    ni.lower = lower; ni.upper = upper; ni.sum = Pair{node_sum[0], node_sum[1]};
    TreeState st{};
    st.m = 1;
    FB_CUDA_CHECK(cudaMemcpyAsync(nodes_[0].p, &ni, sizeof ni, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(state_.p, &st, sizeof st, cudaMemcpyHostToDevice, s_));
    LevelArgs a = level_args(tp);
    set_split_lists(a);
    a.nodes = nodes_[0].as<NodeInfo>();
    a.hist_cur = hist_[0].as<Pair>();
    a.hist_prev = hist_[1].as<Pair>();
    a.last_level = 1;
    launch_split(a, 1, s_);
    FB_CUDA_CHECK(cudaGetLastError());
    SplitRec r;
    last_split_cats_.assign(cat_words_, 0u);
    FB_CUDA_CHECK(cudaMemcpyAsync(&r, node_best_.p, sizeof r, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(last_split_cats_.data(), node_cats_.p, 4ull * cat_words_, cudaMemcpyDeviceToHost,
                                  s_));
    sync();
    const uint32_t* cats = last_split_cats_.data();
    std::memset(out, 0, sizeof *out);
    out->found = r.flags & 1u;
    if (!out->found) return;
    out->feat = r.feat;
    out->missing_left = (r.flags >> 1) & 1u;
    out->categorical = (r.flags >> 2) & 1u;
    out->bin = out->categorical ? 0u : r.bin;  // split.rs:41-51: a categorical split carries its set, bin 0
    out->gain = r.gain;
    out->left_grad = r.left.g; out->left_hess = r.left.h;
    out->right_grad = r.right.g; out->right_hess = r.right.h;
    if (out->categorical) std::memcpy(out->cats, cats, 32);
    else std::fill(last_split_cats_.begin(), last_split_cats_.end(), 0u);
}

void TrainCtx::partition(const uint32_t* rows, uint64_t n, uint32_t feat, uint32_t bin, int missing_left,
                         const uint32_t* cats, uint32_t n_cat_words, uint32_t* out_rows, uint64_t* n_left) {
    ensure_features();
    if (feat >= F_) throw InputError("feature id out of range");
    if (n > n_) throw InputError("more rows than the context holds");
    ensure_tree_buffers(std::max<uint32_t>(buf_depth_, 1), buf_leaves_);
    FB_CUDA_CHECK(cudaMemcpyAsync(rows_[0].p, rows, n * 4, cudaMemcpyHostToDevice, s_));
    NodeInfo ni{};
    ni.start = 0; ni.len = (uint32_t)n; ni.tree_id = 0; ni.parent_slot = -1;
    SplitDesc sd{0, feat, bin, (missing_left ? 2u : 0u) | (cats ? 4u : 0u)};
    if (cats && n_cat_words > cat_words_)
        for (uint32_t w = cat_words_; w < n_cat_words; w++)
            if (cats[w]) throw InputError("the category set holds codes beyond this context's widest feature");
    std::vector<uint32_t> cw(cat_words_, 0u);
    if (cats) std::memcpy(cw.data(), cats, 4ull * std::min(n_cat_words, cat_words_));
    uint32_t cp[2] = {0, ceil_div(n, kChunkRows)};
    TreeState st{};
    st.m = 1; st.chunk_count = cp[1];
    FB_CUDA_CHECK(cudaMemcpyAsync(nodes_[0].p, &ni, sizeof ni, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(split_.p, &sd, sizeof sd, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(node_cats_.p, cw.data(), 4ull * cat_words_, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(chunk_prefix_[0].p, cp, 8, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(state_.p, &st, sizeof st, cudaMemcpyHostToDevice, s_));
    fbgpu_tree_params tp{};
    LevelArgs a = level_args(tp);
    a.nodes = nodes_[0].as<NodeInfo>();
    a.chunk_prefix = chunk_prefix_[0].as<uint32_t>();
    a.rows_cur = rows_[0].as<uint32_t>();
    a.rows_next = rows_[1].as<uint32_t>();
    launch_part_count(a, std::max<uint32_t>(cp[1], 1), s_);
    launch_part_scan(a, s_);
    launch_part_scatter(a, std::max<uint32_t>(cp[1], 1), s_);
    FB_CUDA_CHECK(cudaGetLastError());
    uint32_t nl = 0;
    FB_CUDA_CHECK(cudaMemcpyAsync(&nl, node_left_.p, 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(out_rows, rows_[1].p, n * 4, cudaMemcpyDeviceToHost, s_));
    sync();
    *n_left = nl;
}

// ======================================================================= explain
void make_shap_rule(float* nodes, float* weights) {
    const int n = kShapPoints;
    auto legendre = [](int k, double x) {
        if (k == 0) return 1.0;
        double p0 = 1.0, p1 = x;
        for (int j = 2; j <= k; j++) {
            double jf = (double)j;
            double pk = ((2.0 * jf - 1.0) * x * p1 - (jf - 1.0) * p0) / jf;
            p0 = p1;
            p1 = pk;
        }
        return p1;
    };
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
        nodes[n - 1 - i] = (float)(s * s);
        weights[n - 1 - i] = (float)(2.0 * s * ws);
    }
}

ExplainModel::ExplainModel(int device, uint32_t n_features, uint32_t n_trees, const uint32_t* tree_off,
                           const int32_t* left, const int32_t* right, const uint32_t* feat, const float* value,
                           const uint8_t* flags, const float* hess, const uint32_t* cat_off,
                           const uint32_t* cat_len, const uint32_t* cat_words, uint64_t n_cat_words,
                           float base_margin)
    : device_(device), F_(n_features), T_(n_trees), base_margin_(base_margin) {
    if (n_features == 0 || n_features > 0xffffff) throw InputError("model feature count out of range");
    FB_CUDA_CHECK(cudaSetDevice(device));
    FB_CUDA_CHECK(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking));
    const uint32_t nn = tree_off[n_trees];
    std::vector<DevNode> nodes(std::max<uint32_t>(nn, 1));
    std::vector<uint32_t> coff(std::max<uint32_t>(nn, 1), 0), clen(std::max<uint32_t>(nn, 1), 0);
    double rm_sum = 0.0;
    for (uint32_t t = 0; t < n_trees; t++) {
        const uint32_t a = tree_off[t], b = tree_off[t + 1];
        if (b <= a) throw InputError("every tree has at least one node");
        for (uint32_t i = a; i < b; i++) {
            DevNode d{};
            d.val = value[i];
            d.left = left[i];
            d.right = right[i];
            const uint32_t fl = flags[i] & 7u;
            if (!(fl & 1u)) {
                if (feat[i] >= n_features) throw InputError("split feature out of range");
                if (left[i] <= (int32_t)(i - a) || right[i] <= (int32_t)(i - a) || left[i] >= (int32_t)(b - a) ||
                    right[i] >= (int32_t)(b - a))
                    throw InputError("child index out of range (children must follow their parent)");
            }
            d.meta = (feat[i] & 0xffffffu) | (fl << 24);
            d.hess = hess ? hess[i] : 0.0f;
            nodes[i] = d;
            if (cat_off && (fl & 4u)) {
                coff[i] = cat_off[i];
                clen[i] = cat_len[i];
                if ((uint64_t)cat_off[i] + cat_len[i] > n_cat_words) throw InputError("category set out of range");
            }
        }
        // explain.rs:412-426 root_mean (f64, cover weighted); summed in tree order
        std::vector<double> mean(b - a);
        for (uint32_t i = b; i-- > a;) {
            const DevNode& d = nodes[i];
            if ((d.meta >> 24) & 1u) { mean[i - a] = (double)d.val; continue; }
            double lm = mean[d.left], rmn = mean[d.right];
            if (d.hess == 0.0f) mean[i - a] = 0.5 * (lm + rmn);
            else mean[i - a] = (lm * (double)nodes[a + d.left].hess + rmn * (double)nodes[a + d.right].hess) / (double)d.hess;
        }
        rm_sum += mean[0];
    }
    root_mean_ = (float)rm_sum;
    nodes_.alloc(sizeof(DevNode) * nodes.size());
    tree_off_.alloc(4 * (n_trees + 1));
    cat_off_.alloc(4 * coff.size());
    cat_len_.alloc(4 * clen.size());
    cat_words_.alloc(4 * std::max<uint64_t>(n_cat_words, 1));
    FB_CUDA_CHECK(cudaMemcpyAsync(nodes_.p, nodes.data(), sizeof(DevNode) * nodes.size(), cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(tree_off_.p, tree_off, 4 * (n_trees + 1), cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(cat_off_.p, coff.data(), 4 * coff.size(), cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(cat_len_.p, clen.data(), 4 * clen.size(), cudaMemcpyHostToDevice, s_));
    if (n_cat_words)
        FB_CUDA_CHECK(cudaMemcpyAsync(cat_words_.p, cat_words, 4 * n_cat_words, cudaMemcpyHostToDevice, s_));
    make_shap_rule(rule_nodes_, rule_weights_);
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    h_nodes_ = std::move(nodes);
    h_tree_off_.assign(tree_off, tree_off + n_trees + 1);
    h_coff_ = std::move(coff);
    h_clen_ = std::move(clen);
    if (n_cat_words) h_cat_words_.assign(cat_words, cat_words + n_cat_words);
    dm_.nodes = nodes_.as<DevNode>();
    dm_.tree_off = tree_off_.as<uint32_t>();
    dm_.cat_off = cat_off_.as<uint32_t>();
    dm_.cat_len = cat_len_.as<uint32_t>();
    dm_.cat_words = cat_words_.as<uint32_t>();
    dm_.n_trees = n_trees;
    dm_.n_features = n_features;
}

ExplainModel::~ExplainModel() {
    if (s_) {
        cudaStreamSynchronize(s_);
        cudaStreamDestroy(s_);
    }
}

void ExplainModel::predict_device(const float* X, uint64_t n, float* out, cudaStream_t s) {
    FB_CUDA_CHECK(cudaSetDevice(device_));
    launch_predict(dm_, X, n, base_margin_, out, s);
    FB_CUDA_CHECK(cudaGetLastError());
}

void ExplainModel::shap_device(const float* X, uint64_t n, float* out, cudaStream_t s) {
    FB_CUDA_CHECK(cudaSetDevice(device_));
    // path TreeSHAP unless a model shape needs the node-by-node kernel, or
    // FBGPU_SHAP=dfs asks for it (the reference's exact f32 operation order)
    const char* sel = std::getenv("FBGPU_SHAP");
    const bool dfs = sel && std::string(sel) == "dfs";
    if (!dfs && ShapPaths::smem_bytes(F_) <= 227 * 1024) {
        ensure_paths();
        if (paths_.supported) {
            paths_.launch(X, n, F_, base_margin_, root_mean_, out, s);
            FB_CUDA_CHECK(cudaGetLastError());
            return;
        }
    }
    const uint64_t T = shap_threads(n);
    if (T > scratch_threads_) {
        path_.alloc(4 * T * F_);
        tc_.alloc(4 * T * F_);
        scratch_threads_ = T;
    }
    upload_shap_rule(rule_nodes_, rule_weights_, s);
    launch_shap(dm_, X, n, base_margin_, root_mean_, out, path_.as<float>(), tc_.as<float>(), s);
    FB_CUDA_CHECK(cudaGetLastError());
}

void ExplainModel::ensure_paths() {
    if (paths_built_) return;
    paths_.build(h_nodes_, h_tree_off_.data(), T_, F_, h_coff_, h_clen_, h_cat_words_.data(), rule_nodes_,
                 rule_weights_);
    if (paths_.supported) paths_.upload(s_);
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    paths_built_ = true;
}

uint64_t ExplainModel::explain_width(int kind) const {
    if (kind == 0) return T_;
    if (kind == 1) return (uint64_t)F_ + 1;
    if (kind == 2) return ((uint64_t)F_ + 1) * (F_ + 1);
    throw InputError("explain kind must be 0 (leaf), 1 (approx contributions) or 2 (interactions)");
}

// explain.rs:409-421 fill_node_means: float32, children first, then
// (left mean x left cover + right mean x right cover) / cover.
static float node_means(const std::vector<DevNode>& nodes, uint32_t base, uint32_t i, std::vector<float>& means) {
    const DevNode& d = nodes[base + i];
    float v;
    if ((d.meta >> 24) & kNodeLeaf) {
        v = d.val;
    } else {
        float res = node_means(nodes, base, (uint32_t)d.left, means) * nodes[base + d.left].hess;
        res += node_means(nodes, base, (uint32_t)d.right, means) * nodes[base + d.right].hess;
        v = res / d.hess;
    }
    means[base + i] = v;
    return v;
}

void ExplainModel::explain_device(int kind, const float* X, uint64_t n, float* out, cudaStream_t s) {
    FB_CUDA_CHECK(cudaSetDevice(device_));
    (void)explain_width(kind);
    if (kind == 0) {
        launch_pred_leaf(dm_, X, n, out, s);
    } else if (kind == 1) {
        if (!means_.p) {
            std::vector<float> means(std::max<size_t>(h_nodes_.size(), 1), 0.0f);
            for (uint32_t t = 0; t < T_; t++) node_means(h_nodes_, h_tree_off_[t], 0, means);
            means_.alloc(4 * means.size());
            FB_CUDA_CHECK(cudaMemcpyAsync(means_.p, means.data(), 4 * means.size(), cudaMemcpyHostToDevice, s_));
            FB_CUDA_CHECK(cudaStreamSynchronize(s_));
        }
        launch_pred_approx(dm_, means_.as<float>(), X, n, base_margin_, out, s);
    } else {
        ensure_paths();
        if (!paths_.supported)
            throw InputError("pred_interactions on the device supports at most 14 features on a path");
        paths_.launch_inter(X, n, F_, base_margin_, root_mean_, out, s);
    }
    FB_CUDA_CHECK(cudaGetLastError());
}

void ExplainModel::explain_host(int kind, const float* X, uint64_t n, float* out) {
    const uint64_t w = explain_width(kind);
    x_.alloc(std::max<uint64_t>(n * F_ * 4, 16));
    out_.alloc(std::max<uint64_t>(n * w * 4, 16));
    FB_CUDA_CHECK(cudaMemcpyAsync(x_.p, X, n * F_ * 4, cudaMemcpyHostToDevice, s_));
    explain_device(kind, x_.as<float>(), n, out_.as<float>(), s_);
    FB_CUDA_CHECK(cudaMemcpyAsync(out, out_.p, n * w * 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
}

void ExplainModel::predict_host(const float* X, uint64_t n, float* out) {
    x_.alloc(std::max<uint64_t>(n * F_ * 4, 16));
    out_.alloc(std::max<uint64_t>(n * 4, 16));
    FB_CUDA_CHECK(cudaMemcpyAsync(x_.p, X, n * F_ * 4, cudaMemcpyHostToDevice, s_));
    predict_device(x_.as<float>(), n, out_.as<float>(), s_);
    FB_CUDA_CHECK(cudaMemcpyAsync(out, out_.p, n * 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
}

void ExplainModel::shap_host(const float* X, uint64_t n, float* out) {
    x_.alloc(std::max<uint64_t>(n * F_ * 4, 16));
    out_.alloc(std::max<uint64_t>(n * (F_ + 1) * 4, 16));
    FB_CUDA_CHECK(cudaMemcpyAsync(x_.p, X, n * F_ * 4, cudaMemcpyHostToDevice, s_));
    shap_device(x_.as<float>(), n, out_.as<float>(), s_);
    FB_CUDA_CHECK(cudaMemcpyAsync(out, out_.p, n * (F_ + 1) * 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
}

}  // namespace fbg

// ======================================================================= C ABI
using fbg::ExplainModel;
using fbg::TrainCtx;

struct fbgpu_ctx {
    TrainCtx impl;
    explicit fbgpu_ctx(const fbgpu_config& c) : impl(c) {}
};


namespace {
template <class F> fbgpu_status guard(fbgpu_ctx* ctx, F&& f) {
    try {
        f();
        return FBGPU_OK;
    } catch (const fbg::InputError& e) {
        (ctx ? ctx->impl.err : fbg::g_last_error) = e.what();
        return FBGPU_EINPUT;
    } catch (const fbg::CudaError& e) {
        (ctx ? ctx->impl.err : fbg::g_last_error) = e.what();
        return FBGPU_ECUDA;
    } catch (const fbg::TimeoutError& e) {
        (ctx ? ctx->impl.err : fbg::g_last_error) = e.what();
        return FBGPU_ETIMEOUT;
    } catch (const fbg::NcclError& e) {
        (ctx ? ctx->impl.err : fbg::g_last_error) = e.what();
        return FBGPU_ENCCL;
    } catch (const std::exception& e) {
        (ctx ? ctx->impl.err : fbg::g_last_error) = e.what();
        return FBGPU_EINTERNAL;
    }
}
}  // namespace

extern "C" {

const char* fbgpu_last_error(const fbgpu_ctx* ctx) { return ctx ? ctx->impl.err.c_str() : fbg::g_last_error.c_str(); }

int32_t fbgpu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

fbgpu_status fbgpu_ctx_create(const fbgpu_config* cfg, fbgpu_ctx** out) {
    return guard(nullptr, [&] {
        if (!cfg || !out) throw fbg::InputError("null argument");
        *out = new fbgpu_ctx(*cfg);
    });
}
void fbgpu_ctx_destroy(fbgpu_ctx* ctx) { delete ctx; }

fbgpu_status fbgpu_set_features(fbgpu_ctx* ctx, const uint32_t* n_bins, const uint8_t* width,
                                const uint8_t* categorical) {
    return guard(ctx, [&] { ctx->impl.set_features(n_bins, width, categorical); });
}
fbgpu_status fbgpu_upload_block(fbgpu_ctx* ctx, const uint32_t* feat_ids, uint32_t n_feats, uint32_t width,
                                const void* data) {
    return guard(ctx, [&] { ctx->impl.upload_block(feat_ids, n_feats, width, data); });
}
fbgpu_status fbgpu_set_labels(fbgpu_ctx* ctx, const float* labels, const float* weights,
                              const float* base_margin_rows, float base_margin) {
    return guard(ctx, [&] { ctx->impl.set_labels(labels, weights, base_margin_rows, base_margin); });
}
fbgpu_status fbgpu_upload_and_quantize_gpair(fbgpu_ctx* ctx, const float* gpair, uint64_t sub_threshold, uint64_t seed,
                                             uint64_t tree, double* scales_out, int64_t* root_sum_out) {
    return guard(ctx, [&] {
        ctx->impl.upload_and_quantize(gpair, sub_threshold, seed, tree, scales_out, root_sum_out);
    });
}
fbgpu_status fbgpu_upload_gpair(fbgpu_ctx* ctx, const int64_t* fixed, const double* scales, const int64_t* root_sum) {
    return guard(ctx, [&] { ctx->impl.upload_fixed(fixed, scales, root_sum); });
}
fbgpu_status fbgpu_round_from_exp(fbgpu_ctx* ctx, int32_t objective, const float* host_exp, uint64_t sub_threshold,
                                  uint64_t seed, uint64_t tree, const double* scales) {
    return guard(ctx, [&] { ctx->impl.round_from_exp(objective, host_exp, sub_threshold, seed, tree, scales); });
}
fbgpu_status fbgpu_round_device(fbgpu_ctx* ctx, int32_t objective, int32_t fast, uint64_t sub_threshold,
                                uint64_t seed, uint64_t tree, double* scales_out, int64_t* root_sum_out) {
    return guard(ctx, [&] {
        ctx->impl.round_device(objective, fast, sub_threshold, seed, tree, scales_out, root_sum_out);
    });
}
fbgpu_status fbgpu_set_outputs(fbgpu_ctx* ctx, uint32_t n_classes, const float* class_margins) {
    return guard(ctx, [&] { ctx->impl.set_outputs(n_classes, class_margins); });
}
fbgpu_status fbgpu_multiclass_gradients(fbgpu_ctx* ctx, int32_t fast) {
    return guard(ctx, [&] { ctx->impl.softmax_gradients(fast); });
}
fbgpu_status fbgpu_quantize_class(fbgpu_ctx* ctx, uint32_t cls, uint64_t sub_threshold, uint64_t seed, uint64_t tree,
                                  int32_t fast, double* scales_out, int64_t* root_sum_out) {
    return guard(ctx, [&] {
        if (cls >= ctx->impl.outputs()) throw fbg::InputError("class index out of range");
        ctx->impl.quantize_class(cls, sub_threshold, seed, tree, fast, scales_out, root_sum_out);
    });
}
fbgpu_status fbgpu_set_output_column(fbgpu_ctx* ctx, uint32_t cls) {
    return guard(ctx, [&] {
        if (cls >= ctx->impl.outputs()) throw fbg::InputError("class index out of range");
        ctx->impl.set_pred_column(cls);
    });
}
fbgpu_status fbgpu_build_tree(fbgpu_ctx* ctx, const fbgpu_tree_params* tp, const uint8_t* enabled,
                              fbgpu_tree_out* out) {
    return guard(ctx, [&] {
        if (!tp) throw fbg::InputError("null tree parameters");
        ctx->impl.build_tree(*tp, enabled, out);
    });
}
fbgpu_status fbgpu_download_margins(fbgpu_ctx* ctx, float* out) {
    return guard(ctx, [&] { ctx->impl.download_margins(out); });
}
fbgpu_status fbgpu_histogram(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n_sel, const int64_t* fixed,
                             int64_t* out) {
    return guard(ctx, [&] { ctx->impl.histogram(rows, n_sel, fixed, out); });
}
fbgpu_status fbgpu_eval_split(fbgpu_ctx* ctx, const int64_t* hist, const int64_t* node_sum, const double* scales,
                              const fbgpu_tree_params* tp, float lower, float upper, const uint8_t* enabled,
                              fbgpu_split* out) {
    return guard(ctx, [&] { ctx->impl.eval_split(hist, node_sum, scales, *tp, lower, upper, enabled, out); });
}
fbgpu_status fbgpu_partition(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n, uint32_t feat, uint32_t bin,
                             int32_t missing_left, const uint32_t* cats, uint32_t* out_rows, uint64_t* n_left) {
    return guard(ctx, [&] { ctx->impl.partition(rows, n, feat, bin, missing_left, cats, 8, out_rows, n_left); });
}
fbgpu_status fbgpu_partition_set(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n, uint32_t feat, int32_t missing_left,
                                 const uint32_t* cats, uint32_t n_words, uint32_t* out_rows, uint64_t* n_left) {
    return guard(ctx, [&] {
        if (!cats) throw fbg::InputError("a category set is required");
        ctx->impl.partition(rows, n, feat, 0, missing_left, cats, n_words, out_rows, n_left);
    });
}
uint32_t fbgpu_ctx_cat_words(const fbgpu_ctx* ctx) { return ctx ? ctx->impl.cat_words() : 0u; }
fbgpu_status fbgpu_split_cats(fbgpu_ctx* ctx, uint32_t* out, uint32_t n_words) {
    return guard(ctx, [&] {
        const std::vector<uint32_t>& c = ctx->impl.last_split_cats();
        for (uint32_t w = 0; w < n_words; w++) out[w] = w < c.size() ? c[w] : 0u;
        for (size_t w = n_words; w < c.size(); w++)
            if (c[w]) throw fbg::InputError("the category set needs fbgpu_ctx_cat_words words");
    });
}

uint64_t fbgpu_launch_count(void) { return fbg::g_launches.load(std::memory_order_relaxed); }

fbgpu_status fbgpu_nccl_unique_id(uint8_t* out) {
    return guard(nullptr, [&] { fbg::nccl_unique_id(out); });
}

fbgpu_status fbgpu_comm_begin(const uint8_t* unique_id, int32_t nranks, int32_t rank, int32_t device,
                              uint32_t timeout_ms, fbgpu_comm** out) {
    return guard(nullptr, [&] {
        if (!unique_id || !out) throw fbg::InputError("unique_id and out must not be null");
        if (nranks < 2 || rank < 0 || rank >= nranks) throw fbg::InputError("invalid rank / world size");
        auto pc = std::make_unique<fbgpu_comm>();
        pc->impl.nranks = nranks;
        pc->impl.rank = rank;
        pc->impl.comm.reset(new fbg::NcclComm(unique_id, nranks, rank, device, timeout_ms, false));
        fbg::PendingComm* p = &pc->impl;
        p->worker = std::thread([p, device] {
            try {
                FB_CUDA_CHECK(cudaSetDevice(device));
                p->comm->wait_init();
                // the first collectives of each size set up NCCL's connections;
                // run a small and a histogram-sized one now, on every rank
                cudaStream_t st = nullptr;
                FB_CUDA_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
                struct Owner {
                    cudaStream_t s;
                    ~Owner() { cudaStreamDestroy(s); }
                } owner{st};
                fbg::DevMem buf;
                buf.alloc(8u << 20);
                FB_CUDA_CHECK(cudaMemsetAsync(buf.p, 0, 8u << 20, st));
                p->comm->allreduce(buf.p, buf.p, 2, true, false, st);
                p->comm->allreduce(buf.p, buf.p, (8u << 20) / 8, true, false, st);
                p->comm->sync(st);
            } catch (...) {
                p->error = std::current_exception();
            }
        });
        *out = pc.release();
    });
}

void fbgpu_comm_free(fbgpu_comm* c) { delete c; }

int32_t fbgpu_comm_usable(fbgpu_comm* c) {
    if (!c) return 0;
    if (c->impl.worker.joinable()) return 0;  // still starting: not yet joined by any context
    return c->impl.usable() ? 1 : 0;
}

void fbgpu_comm_abort(fbgpu_comm* c) {
    if (c && !c->impl.worker.joinable() && c->impl.comm) c->impl.comm->abort();
}

fbgpu_status fbgpu_ctx_adopt_comm(fbgpu_ctx* ctx, fbgpu_comm* c) {
    return guard(ctx, [&] {
        if (!c) throw fbg::InputError("null communicator");
        ctx->impl.adopt_comm(c->impl.share(), c->impl.nranks, c->impl.rank);
    });
}

fbgpu_status fbgpu_ctx_set_comm(fbgpu_ctx* ctx, const uint8_t* unique_id, int32_t nranks, int32_t rank,
                                uint32_t timeout_ms) {
    return guard(ctx, [&] { ctx->impl.set_comm(unique_id, nranks, rank, timeout_ms); });
}

int32_t fbgpu_exact_exp_available(const char** why) {
    const auto& t = fbg::exp_table();
    if (why) *why = t.ok ? "" : t.why.c_str();
    return t.ok ? 1 : 0;
}

fbgpu_status fbgpu_expf_check(int32_t device, uint32_t begin, uint32_t count, uint64_t* mismatches,
                              uint32_t* report) {
    return guard(nullptr, [&] {
        const auto& t = fbg::exp_table();
        if (!t.ok) throw fbg::InputError(t.why);
        FB_CUDA_CHECK(cudaSetDevice(device));
        fbg::DevMem tab, out;
        tab.alloc(sizeof(uint2) * t.slots.size());
        out.alloc(4ull * std::max<uint32_t>(count, 1));
        FB_CUDA_CHECK(cudaMemcpy(tab.p, t.slots.data(), sizeof(uint2) * t.slots.size(), cudaMemcpyHostToDevice));
        fbg::launch_expf_emulate(tab.as<uint2>(), t.probes, begin, count, out.as<uint32_t>(), nullptr);
        std::vector<uint32_t> dev(count);
        FB_CUDA_CHECK(cudaMemcpy(dev.data(), out.p, 4ull * count, cudaMemcpyDeviceToHost));
        uint64_t bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
        for (int64_t i = 0; i < (int64_t)count; i++) {
            const uint32_t key = begin + (uint32_t)i;
            float x;
            std::memcpy(&x, &key, 4);
            const float g = expf(x);
            uint32_t gb;
            std::memcpy(&gb, &g, 4);
            float d;
            std::memcpy(&d, &dev[i], 4);
            if (gb != dev[i] && !(std::isnan(g) && std::isnan(d))) bad++;
        }
        *mismatches = bad;
        if (report && bad) {  // first mismatches: (input, host expf, device, host fexp_core) x 4
            int k = 0;
            for (uint32_t i = 0; i < count && k < 4; i++) {
                const uint32_t key = begin + i;
                float x;
                std::memcpy(&x, &key, 4);
                const float g = expf(x);
                uint32_t gb;
                std::memcpy(&gb, &g, 4);
                float d;
                std::memcpy(&d, &dev[i], 4);
                if (gb != dev[i] && !(std::isnan(g) && std::isnan(d))) {
                    const float m = fbx::fexp_core(x);
                    uint32_t mb;
                    std::memcpy(&mb, &m, 4);
                    report[4 * k] = key; report[4 * k + 1] = gb; report[4 * k + 2] = dev[i]; report[4 * k + 3] = mb;
                    k++;
                }
            }
        }
    });
}

fbgpu_status fbgpu_model_create(int32_t device, uint32_t n_features, uint32_t n_trees, const uint32_t* tree_off,
                                const int32_t* left, const int32_t* right, const uint32_t* feat, const float* value,
                                const uint8_t* flags, const float* hess, const uint32_t* cat_off,
                                const uint32_t* cat_len, const uint32_t* cat_words, uint64_t n_cat_words,
                                float base_margin, fbgpu_model** out) {
    return guard(nullptr, [&] {
        if (!out || !tree_off) throw fbg::InputError("null argument");
        *out = new fbgpu_model(device, n_features, n_trees, tree_off, left, right, feat, value, flags, hess, cat_off,
                               cat_len, cat_words, n_cat_words, base_margin);
    });
}
void fbgpu_model_destroy(fbgpu_model* m) { delete m; }
fbgpu_status fbgpu_predict(fbgpu_model* m, const float* X, uint64_t n, float* out) {
    return guard(nullptr, [&] { m->impl.predict_host(X, n, out); });
}
fbgpu_status fbgpu_predict_device(fbgpu_model* m, const float* X, uint64_t n, float* out, void* stream) {
    return guard(nullptr, [&] { m->impl.predict_device(X, n, out, (cudaStream_t)stream); });
}
fbgpu_status fbgpu_shap(fbgpu_model* m, const float* X, uint64_t n, float* out) {
    return guard(nullptr, [&] { m->impl.shap_host(X, n, out); });
}
fbgpu_status fbgpu_shap_device(fbgpu_model* m, const float* X, uint64_t n, float* out, void* stream) {
    return guard(nullptr, [&] { m->impl.shap_device(X, n, out, (cudaStream_t)stream); });
}
fbgpu_status fbgpu_explain(fbgpu_model* m, int32_t kind, const float* X, uint64_t n, float* out) {
    return guard(nullptr, [&] { m->impl.explain_host(kind, X, n, out); });
}
fbgpu_status fbgpu_explain_device(fbgpu_model* m, int32_t kind, const float* X, uint64_t n, float* out,
                                  void* stream) {
    return guard(nullptr, [&] { m->impl.explain_device(kind, X, n, out, (cudaStream_t)stream); });
}

}  // extern "C"
