// Host side of the training context and the explanation model (C++ classes
// behind the C ABI in include/fbgpu.h).
#pragma once
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <exception>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "nccl_loader.h"

#include "../../include/fbgpu.h"
#include "explain_kernels.cuh"
#include "train_kernels.cuh"

namespace fbg {

inline uint32_t ceil_div(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

struct CudaError : std::runtime_error {
    CudaError(cudaError_t e, const char* what, const char* file, int line)
        : std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(e) + " in " + what + " (" + file + ":" +
                             std::to_string(line) + ")") {}
};
struct InputError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Device blocks through the process-wide cache (devmem.cu): dev_alloc
// returns a block of at least n bytes and its size in *cap; dev_free takes
// the block back once its device is idle.
void* dev_alloc(size_t n, size_t* cap);
void dev_free(void* p, size_t cap);
void* pinned_alloc(size_t n, size_t* cap);
void pinned_free(void* p, size_t cap);

// Captures the work a stream is given while `on` (end() returns the graph);
// a capture left open by an exception is ended and discarded.
struct CaptureGuard {
    cudaStream_t s;
    bool on;
    CaptureGuard(cudaStream_t st, bool enable) : s(st), on(false) {
        if (enable) begin();
    }
    void begin() {
        FB_CUDA_CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
        on = true;
    }
    cudaGraph_t end() {
        cudaGraph_t g = nullptr;
        on = false;
        FB_CUDA_CHECK(cudaStreamEndCapture(s, &g));
        return g;
    }
    ~CaptureGuard() {
        if (!on) return;
        cudaGraph_t g = nullptr;
        if (cudaStreamEndCapture(s, &g) == cudaSuccess && g) cudaGraphDestroy(g);
        (void)cudaGetLastError();
    }
    CaptureGuard(const CaptureGuard&) = delete;
    CaptureGuard& operator=(const CaptureGuard&) = delete;
};

// Owning device allocation; `bytes` is the size asked for.
struct DevMem {
    void* p = nullptr;
    size_t bytes = 0, cap = 0;
    DevMem() = default;
    DevMem(const DevMem&) = delete;
    DevMem& operator=(const DevMem&) = delete;
    ~DevMem() { release(); }
    void release() {
        if (p) dev_free(p, cap);
        p = nullptr;
        bytes = cap = 0;
    }
    void alloc(size_t n) {
        release();
        if (n == 0) n = 16;
        p = dev_alloc(n, &cap);
        bytes = n;
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

// Pinned host buffer through the same cache; `bytes` is its capacity.
struct PinnedMem {
    void* p = nullptr;
    size_t bytes = 0;
    PinnedMem() = default;
    PinnedMem(const PinnedMem&) = delete;
    PinnedMem& operator=(const PinnedMem&) = delete;
    ~PinnedMem() { release(); }
    void release() {
        if (p) pinned_free(p, bytes);
        p = nullptr;
        bytes = 0;
    }
    void reserve(size_t n) {
        if (n <= bytes) return;
        release();
        p = pinned_alloc(n, &bytes);
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

class TrainCtx {
   public:
    explicit TrainCtx(const fbgpu_config& cfg);
    ~TrainCtx();

    void set_features(const uint32_t* n_bins, const uint8_t* width, const uint8_t* categorical);
    void upload_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width, const void* data);
    // A block already quantized on this device as row records (`stride`
    // bytes, zero padded, n_rows + 16 B); the caller keeps it alive for the
    // context's lifetime.
    void adopt_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width, const uint8_t* records,
                     uint32_t stride);
    void set_labels(const float* labels, const float* weights, const float* base_rows, float base_margin);

    // Round start variants; each leaves the fixed gradients, the root sum
    // and the scales on the device.
    void upload_and_quantize(const float* gpair, uint64_t th, uint64_t seed, uint64_t tree, double* scales_out,
                             int64_t* sum_out);
    void upload_fixed(const int64_t* fixed, const double* scales, const int64_t* sum);
    void round_from_exp(int objective, const float* host_exp, uint64_t th, uint64_t seed, uint64_t tree,
                        const double* scales);
    void round_device(int objective, int fast, uint64_t th, uint64_t seed, uint64_t tree, double* scales_out,
                      int64_t* sum_out);
    // The parameters of the round_device call that will follow the next
    // launched tree.  When that tree ends with the tree walk, the walk also
    // computes that round's gradient pairs and bounds from the new margins,
    // and the matching round_device call starts at its scales.  Applies to
    // one output, squared error or logistic, with gradients on the device.
    void set_next_gradient(int objective, int fast, uint64_t th, uint64_t seed, uint64_t tree);

    void build_tree(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* out);
    // A tree in two halves, for trees that need no host decision while they
    // grow (depthwise, and lossguide whose cap cannot bind): launch enqueues
    // the tree and the copy of its result into a pinned slot and returns;
    // collect waits for the oldest launched tree and fills `out`.  Two slots:
    // a caller can launch the next round's gradients and tree before it
    // collects this one, so the host's work between rounds overlaps the
    // device's.  build_tree() is launch + collect.
    bool tree_async(const fbgpu_tree_params& tp) const;
    void build_tree_launch(const fbgpu_tree_params& tp, const uint8_t* enabled);
    void build_tree_collect(fbgpu_tree_out* out);
    uint32_t trees_in_flight() const { return slots_pending_; }
    // Waits for the stream and drops the launched trees (after an error).
    void abandon_trees() {
        slots_pending_ = 0;
        scale_err_pending_ = false;
        next_grad_.set = fused_grad_.set = false;
        sync();
    }

    // Multiclass (multi:softprob / multi:softmax, training/mod.rs:2564-2800):
    // K margin columns, class-major, each starting at its class's base margin.
    void set_outputs(uint32_t K, const float* class_margins);
    uint32_t outputs() const { return K_; }
    // objective.rs:1175-1219 softmax gradients of all K classes from the
    // current margins (the host expf reproduced on the device unless fast).
    void softmax_gradients(int fast);
    // Class k's column: sampling mask keyed by `tree`, bounds, scales (host
    // libm, or the device in fast mode), fixed point and root sum.
    void quantize_class(uint32_t k, uint64_t th, uint64_t seed, uint64_t tree, int fast, double* scales_out = nullptr,
                        int64_t* sum_out = nullptr);
    // The margin column the next build_tree adds its leaf values to.
    void set_pred_column(uint32_t k) {
        pred_col_ = k;
        next_grad_.set = fused_grad_.set = false;
    }

    // Row sharding over several GPUs: one context per GPU, one NCCL
    // communicator per context (ranks in the same order on every GPU).
    void set_comm(const uint8_t* unique_id, int nranks, int rank, uint32_t timeout_ms);
    // A communicator initialized ahead of time (fbgpu_comm_begin).
    void adopt_comm(std::shared_ptr<NcclComm> comm, int nranks, int rank);
    int nranks() const { return nranks_; }
    // Waits for the training stream; when sharded, a bounded poll that aborts
    // the communicator if a peer stops answering.
    void sync();
    // Max over ranks of non-negative host doubles (bit patterns order like the values).
    void allreduce_max_host(double* v, int count);
    void download_margins(float* out);

    void histogram(const uint32_t* rows, uint64_t n_sel, const int64_t* fixed, int64_t* out);
    void eval_split(const int64_t* hist, const int64_t* node_sum, const double* scales, const fbgpu_tree_params& tp,
                    float lower, float upper, const uint8_t* enabled, fbgpu_split* out);
    // cats: n_cat_words words (NULL: numeric split); words beyond them are zero
    void partition(const uint32_t* rows, uint64_t n, uint32_t feat, uint32_t bin, int missing_left,
                   const uint32_t* cats, uint32_t n_cat_words, uint32_t* out_rows, uint64_t* n_left);
    // Words of a category set in this context: 8, or enough for the widest
    // categorical feature (a bit per code).
    uint32_t cat_words() const { return cat_words_; }
    // The full category set of the last eval_split (cat_words() words).
    const std::vector<uint32_t>& last_split_cats() const { return last_split_cats_; }

    // Internal access for the engine (same library).
    cudaStream_t stream() const { return s_; }
    float* dev_margins() const { return pred_.as<float>(); }
    uint64_t n_local() const { return n_; }
    const fbgpu_config& config() const { return cfg_; }
    float last_tree_ms() const { return last_tree_ms_; }
    // Exact logistic gradients can run on the device (verified host-expf table).
    bool has_exact_exp() const { return exptab_.p != nullptr; }
    // Histogram-phase statistics of the trees grown since the last reset
    // (enabled by set_stats): device time, launches and algorithmic bytes
    // (rows x (bin bytes + 16 B gradient + 4 B row id) + bins x 16 B flushed).
    void set_stats(bool on) { stats_ = on; }
    void reset_stats() { hist_ms_ = 0; hist_launches_ = 0; hist_bytes_ = 0; comm_ms_ = 0; hist_updates_ = 0; }
    // (row, feature) histogram updates of those trees
    double hist_updates() const { return hist_updates_; }
    double hist_ms() const { return hist_ms_; }
    // Of hist_ms: the device time of the per-level histogram all-reduces (sharded contexts).
    double comm_ms() const { return comm_ms_; }
    double hist_launches() const { return hist_launches_; }
    double hist_bytes() const { return hist_bytes_; }

    std::string err;

   private:
    struct Block {
        std::vector<uint32_t> feats;  // global ids, ascending
        uint32_t width = 2;
        uint32_t stride = 0;
        DevMem data;                   // owned records (upload_block)
        const uint8_t* base = nullptr; // records read by the kernels (owned or adopted)
        DevMem cols;                   // column-major copy read by the partition passes
    };
    std::unique_ptr<Block> new_block(const uint32_t* feat_ids, uint32_t n_feats, uint32_t width);
    void register_block(std::unique_ptr<Block> b);
    void ensure_features() const;
    void plan_tiles(const uint8_t* enabled, bool rank_major = false);
    void launch_histograms(const uint32_t* rows, const NodeInfo* nodes, const uint32_t* acc_list,
                           const unsigned long long* acc_prefix, uint64_t rows_upper, Pair* out = nullptr,
                           unsigned long long slot = 0);
    // Feature-sharded split search of a row-sharded depthwise tree: feature
    // ranges per rank (balanced by bins), this rank's range and block size.
    void setup_split_shards();
    void ensure_tree_buffers(uint32_t max_depth, uint32_t max_leaves, bool lossguide = false);
    void ensure_lossguide_buffers(uint32_t max_leaves);
    void build_tree_lossguide(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* out);
    // the launch half; a best-first tree is grown and read back into lg_out here
    void build_tree_launch(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* lg_out);
    LevelArgs level_args(const fbgpu_tree_params& tp) const;
    void set_split_lists(LevelArgs& a);
    DevMem d_split_lists_;  // [numeric features of <= 256 bins | the rest] of the cached range
    std::vector<uint32_t> split_lists_host_;
    uint32_t split_lists_lo_ = ~0u, split_lists_hi_ = ~0u, n_split_num_ = 0, n_split_cta_ = 0;
    GradArgs grad_args() const;

    fbgpu_config cfg_;
    cudaStream_t s_ = nullptr;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    uint64_t n_ = 0;
    uint32_t F_ = 0;
    std::vector<uint32_t> nbins_, hoff_;
    std::vector<uint8_t> width_, cat_;
    uint64_t total_bins_ = 0;
    std::vector<std::unique_ptr<Block>> blocks_;
    std::vector<int> feat_block_;
    std::vector<uint32_t> feat_byte_;
    bool has_cat_ = false;
    uint32_t cat_words_ = 8, n_cat_ = 0;  // set width (words) and categorical feature count
    std::vector<uint32_t> cat_slot_;      // per feature: index among the categorical features
    std::vector<uint32_t> last_split_cats_;

    // feature tables
    DevMem d_hoff_, d_floc_, d_floc_rec_, d_enabled_, d_mono_, d_cat_, d_cat_slot_;
    std::vector<uint8_t> last_enabled_;
    std::vector<int8_t> last_mono_;
    bool tiles_valid_ = false;
    bool tiles_rank_major_ = false;  // the plan's packed bin indices carry ranks (feature-sharded split search)
    DevMem d_tiles_, d_tfeat_;
    uint32_t tile_off_gen_[2] = {0, 0}, n_gen_[2] = {0, 0}, tile_off_lpf_[2] = {0, 0}, n_lpf_[2] = {0, 0};
    size_t tile_smem_ = 0, tile_smem_lpf_ = 0, tile_smem_stage_ = 0;
    int hist_stages_ = 0;  // staged lane-per-feature histogram: cp.async stages, 0 = unstaged kernel
    uint32_t tile_off_wide_ = 0, n_wide_ = 0;  // wide tiles (8 lanes per row)
    uint64_t tile_bins_gen_[2] = {0, 0}, tile_bins_lpf_[2] = {0, 0}, tile_bins_wide_ = 0,
             tile_bins_direct_[2] = {0, 0};  // mean bins per tile of each launch
    uint32_t tile_off_direct_[2] = {0, 0}, n_direct_[2] = {0, 0};  // global-atomic tiles (no shared histogram)
    size_t tile_smem_wide_ = 0;
    int wide_stages_ = 4;
    int smem_budget_ = 0;

    // rows / gradients
    DevMem label_, weight_, pred_, gpair_f32_, host_exp_, fixed_;
    uint32_t K_ = 1, pred_col_ = 0;  // margin columns (classes) and the one the tree updates
    struct NextGrad {
        bool set = false;
        int objective = 0, fast = 0;
        uint64_t th = 0, seed = 0, tree = 0;
        bool same(int o, int f, uint64_t t, uint64_t s, uint64_t r) const {
            return set && objective == o && fast == f && th == t && seed == s && tree == r;
        }
    };
    NextGrad next_grad_;   // for the next launched tree's walk
    NextGrad fused_grad_;  // the round whose gradients the last tree's walk computed
    DevMem gp_multi_;                 // multiclass: K x n f32 gradient pairs of the round
    DevMem sums_;  // [0..1] root sum, [2..3] max bits, [4..5] scales (double), [6] scale error word
    // exact scales on the device: the row count's exception list (qscale.h)
    DevMem d_scale_exc_;
    uint32_t n_scale_exc_ = 0;
    uint64_t scale_exc_rows_ = ~0ull;
    bool scale_err_pending_ = false;  // a device scale kernel ran; its error word is checked at the next readback
    void launch_scales(const unsigned long long* maxbits, bool fast);
    void check_scale_error(const unsigned long long* host_err);
    void read_scales_sum(double* scales_out, int64_t* sum_out);
    DevMem exptab_;  // host-expf exception table (fexp.h), empty when unverified
    std::shared_ptr<NcclComm> comm_;
    int nranks_ = 1, rank_ = 0;
    DevMem node_left_global_, comm_scratch_;
    // feature-sharded split search (row-sharded depthwise trees): rank r
    // scores features [rank_feat_lo_[r], rank_feat_lo_[r + 1]) whose bins are
    // [rank_bin_lo_[r], rank_bin_lo_[r + 1]); a rank's block holds chunk_pairs_
    // pairs per accumulate slot
    bool split_shard_ = false;
    std::vector<uint32_t> rank_feat_lo_, rank_bin_lo_, feat_rank_;
    uint64_t chunk_pairs_ = 0;
    DevMem hist_rs_, best_all_, cats_all_;
    PinnedMem h_stride_;
    void allreduce_u64(void* buf, size_t count, bool max_op);
    void allreduce_u32(const void* src, void* dst, size_t count);
    void reduce_root_sum(bool now);
    bool root_pending_ = false;  // sharded: this round's root sum is still rank-local
    uint32_t exp_probes_ = 0;
    bool has_weight_ = false;
    PinnedMem h_stage_;

    // tree buffers
    uint32_t buf_depth_ = 0xffffffffu, buf_leaves_ = 0xffffffffu;
    bool buf_lossguide_ = false;
    // best-first growth (lossguide.cu): slot table, wave descriptors, final leaves
    DevMem lg_slots_, lg_slot_hist_, lg_slot_best_, lg_slot_cats_, lg_wave_, lg_wave_out_, lg_eval_slot_,
        lg_node_hist_, lg_final_slot_, lg_final_value_;
    PinnedMem h_lg_;
    uint32_t lg_leaves_ = 0xffffffffu, lg_kmax_ = 0, lg_slot_cap_ = 0, lg_hist_cap_ = 0;
    uint32_t max_level_nodes_ = 0, max_split_nodes_ = 0, max_acc_ = 0, max_tree_nodes_ = 0, max_chunks_ = 0;
    DevMem rows_[2], nodes_[2], acc_list_[2], acc_prefix_[2], chunk_prefix_[2];
    DevMem dirflags_, hist_acc_, hist_[2], feat_best_, feat_cats_, node_best_, node_cats_, split_, chunk_left_, chunk_off_,
        node_left_, trec_, tcats_, state_;
    // readback slots of launched depthwise trees (build_tree_launch / _collect)
    struct ReadSlot {
        PinnedMem tree;   // TreeRec[max_tree_nodes_] | category sets | TreeState
        PinnedMem small;  // 16 levels x 16 B of level statistics, then the scale error word
        cudaEvent_t ev0 = nullptr, ev1 = nullptr, done = nullptr;  // tree start, tree end, readback copied
        cudaEvent_t hev[32] = {}, hevc[16] = {};
        bool lossguide = false, stats = false, scale_err = false;
        uint32_t maxd = 0, W = 8, max_nodes = 0;
        double launches_per_level = 0, row_bytes = 0, bins = 0, feats = 0;  // statistics of the launch's plan
    };
    ReadSlot slot_[2];
    uint32_t slot_next_ = 0, slots_pending_ = 0;  // the oldest pending slot is (slot_next_ + 2 - pending) % 2
    void wait_event(cudaEvent_t ev);
    // per readback slot and graph segment (one per level's span between two
    // collectives when sharded, else one per tree): the last captured
    // executable graph
    static constexpr int kTreeSegments = 17;
    cudaGraphExec_t tree_exec_[2][kTreeSegments] = {};
    void launch_graph(cudaGraph_t g, int slot, int segment);
    PinnedMem h_small_;  // 512 B of pinned readback: no pageable copy waits behind a collective
    float last_tree_ms_ = 0.0f;
    bool stats_ = false;
    DevMem level_stats_;
    DevMem fuse_;  // last-CTA counters of the fused level kernels (depthwise)
    DevMem part_cnt_;  // k_part_level reservation counters, zero between levels
    double hist_ms_ = 0, hist_launches_ = 0, hist_bytes_ = 0, comm_ms_ = 0, hist_updates_ = 0;
};

// Root-to-leaf path form of a model's trees for the path TreeSHAP kernel
// (shap_paths.cu): per path element the feature's condition and the
// row-independent quadrature factors.
struct ShapPaths {
    int M = 4, KMAX = 8;              // quadrature points, features per path (kernel template)
    bool supported = false;           // false: a path the kernel cannot represent (use the DFS kernel)
    uint32_t n_elems = 0;
    uint32_t mask_words = 8;          // words of a category mask (a bit per code)
    std::vector<uint32_t> words, chunk_off, masks;
    DevMem d_words, d_chunks, d_masks;
    mutable DevMem d_acc;             // k_shap_paths: per-CTA f64 totals of phi
    void build(const std::vector<DevNode>& nodes, const uint32_t* tree_off, uint32_t n_trees, uint32_t F,
               const std::vector<uint32_t>& cat_off, const std::vector<uint32_t>& cat_len, const uint32_t* cat_words,
               const float* rule_nodes, const float* rule_weights);
    void upload(cudaStream_t s);
    static size_t smem_bytes(uint32_t F);
    void launch(const float* X, uint64_t n, uint32_t F, float bias, float root_mean, float* out, cudaStream_t s) const;
    // SHAP interaction values over the same paths (warp per row)
    float rule_w8[8] = {};
    DevMem d_rule_w;
    DevMem d_inter_scratch;           // interactions of models too wide for a shared-memory matrix
    static size_t inter_smem_bytes(uint32_t F, uint32_t warps);
    static uint32_t inter_warps(uint32_t F);
    void launch_inter(const float* X, uint64_t n, uint32_t F, float bias, float root_mean, float* out, cudaStream_t s);
};

class ExplainModel {
   public:
    ExplainModel(int device, uint32_t n_features, uint32_t n_trees, const uint32_t* tree_off, const int32_t* left,
                 const int32_t* right, const uint32_t* feat, const float* value, const uint8_t* flags,
                 const float* hess, const uint32_t* cat_off, const uint32_t* cat_len, const uint32_t* cat_words,
                 uint64_t n_cat_words, float base_margin);
    ~ExplainModel();
    void predict_device(const float* X, uint64_t n, float* out, cudaStream_t s);
    void shap_device(const float* X, uint64_t n, float* out, cudaStream_t s);
    void predict_host(const float* X, uint64_t n, float* out);
    void shap_host(const float* X, uint64_t n, float* out);
    // explain.rs Kind::Leaf (0), Contribs { approx: true } (1), Interactions (2)
    void explain_device(int kind, const float* X, uint64_t n, float* out, cudaStream_t s);
    void explain_host(int kind, const float* X, uint64_t n, float* out);
    uint64_t explain_width(int kind) const;
    uint32_t n_features() const { return F_; }
    cudaStream_t stream() const { return s_; }

   private:
    int device_;
    uint32_t F_, T_;
    float base_margin_, root_mean_;
    DevMem nodes_, tree_off_, cat_off_, cat_len_, cat_words_, path_, tc_, x_, out_;
    uint64_t scratch_threads_ = 0;
    cudaStream_t s_ = nullptr;
    DevModel dm_{};
    float rule_nodes_[kShapPoints], rule_weights_[kShapPoints];
    // host copy of the trees for the path form, built at the first SHAP call
    std::vector<DevNode> h_nodes_;
    std::vector<uint32_t> h_tree_off_, h_coff_, h_clen_, h_cat_words_;
    ShapPaths paths_;
    bool paths_built_ = false;
    void ensure_paths();
    DevMem means_;  // Saabas per-node means (explain.rs:409-421), built at the first approx call
};

// A communicator whose initialization, and a warm-up of the collectives the
// training will use, run on a background host thread while the caller
// prepares its data (fbgpu_comm_begin).  take() waits for it.
struct PendingComm {
    std::shared_ptr<NcclComm> comm;
    std::thread worker;
    std::exception_ptr error;
    int nranks = 1, rank = 0;
    ~PendingComm() {
        if (worker.joinable()) worker.join();
    }
    // The communicator, shared with the context that joins it; the handle
    // keeps its reference, so a later context can join it again.
    std::shared_ptr<NcclComm> share() {
        if (worker.joinable()) worker.join();
        if (error) std::rethrow_exception(error);
        if (!comm || comm->failed()) throw NcclError("the communicator failed or was aborted");
        return comm;
    }
    // Started without error, not failed, and no context holds it.
    bool usable() const { return !worker.joinable() && !error && comm && !comm->failed() && comm.use_count() == 1; }
};

// Sets the message fbgpu_last_error(NULL) returns on this thread.
void noalloc_set_error(const char* msg);

// explain.rs:141-169 endpoint-squared Gauss-Legendre rule (f64, stored as f32).
void make_shap_rule(float* nodes, float* weights);

// types.rs:366-385 pow2_scale with the host libm (exact mode).
double pow2_scale_host(double max_abs, uint64_t n_rows);
// The f32 bounds whose reference scale is not 2^(binary exponent of raw) for
// n_rows rows, sorted (qscale.h).
std::vector<fbx::ScaleExc> build_scale_exceptions(uint64_t n_rows);

}  // namespace fbg

// The C ABI's early communicator handle (include/fbgpu.h fbgpu_comm).
struct fbgpu_comm {
    fbg::PendingComm impl;
};

// The C ABI's explanation-model handle (include/fbgpu.h fbgpu_model).
struct fbgpu_model {
    fbg::ExplainModel impl;
    template <class... A> explicit fbgpu_model(A&&... a) : impl(std::forward<A>(a)...) {}
};
