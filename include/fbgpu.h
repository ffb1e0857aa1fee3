/*
 * fbgpu.h — C ABI of the FerrisBoost B200 engine (libfbgpu.so).
 *
 * Plain pointers, sizes and status codes; no C++ types cross the boundary and
 * no exception leaves it.  Every entry point returns an fbgpu_status; the
 * message of the last failure is available from fbgpu_last_error(ctx) or,
 * for failures without a context, fbgpu_last_error(NULL) (thread local).
 *
 * Entry points are grouped as the reference's CUDA backend boundary
 * (mdai001/FerrisBoost src/backend/mod.rs, the cfg-swapped stub whose
 * signatures the Rust training engine calls) plus the explanation models
 * (src/backend/cuda/explain.rs, src/backend/cuda/inference.rs) and the
 * engine-level calls the Python package uses.  Each declaration cites the
 * reference interface it replaces.
 *
 * Layout contracts:
 *   - gradient pairs are interleaved [grad, hess] per row (types.rs:101-107
 *     GradPair as f32, types.rs:151-175 GradPairFixed as int64);
 *   - a column block is column-major, data[local_feat * n_rows + row]
 *     (data/columns.rs:9-25), 1 or 2 bytes per bin, missing = 255 / 65535;
 *   - histograms are total_bins int64 pairs, features in ascending global
 *     order, feature f at offsets[f] (data/columns.rs:270-279).
 */
#ifndef FBGPU_H
#define FBGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  INPUT maps to Python ValueError and the others to
 * RuntimeError, as the reference's InputError split does (src/error.rs:1-70). */
typedef enum fbgpu_status {
    FBGPU_OK = 0,
    FBGPU_EINPUT = 1,
    FBGPU_ECUDA = 2,
    FBGPU_ENCCL = 3,
    FBGPU_ETIMEOUT = 4,
    FBGPU_EINTERNAL = 5
} fbgpu_status;

typedef struct fbgpu_ctx fbgpu_ctx;
typedef struct fbgpu_model fbgpu_model;

/* Context shape.  Replaces GpuTrainCtx::new_with_shape
 * (src/backend/mod.rs:245-255): every device buffer of a training run is
 * allocated here, none during training (src/training/mod.rs:1708-1714). */
typedef struct fbgpu_config {
    int32_t device;
    uint32_t n_features;
    uint64_t n_rows;          /* rows held by this context (its shard) */
    uint64_t n_rows_global;   /* rows over all ranks (quantizer budget) */
    uint64_t row_offset;      /* global index of this shard's first row */
    uint32_t max_depth;       /* 0..=14 (types.rs:424 MAX_DEPTH_LIMIT) */
    uint32_t max_leaves;      /* 0 = unlimited */
    uint32_t hist_smem_bytes; /* shared-memory budget of a histogram tile; 0 = default */
    int32_t gpu_math;         /* 0 exact, 1 fast (types.rs:80-87 GpuMath) */
} fbgpu_config;

/* Per-tree split parameters (TrainParams, types.rs:433-686). */
typedef struct fbgpu_tree_params {
    float eta;
    float lambda;
    float gamma;
    float min_child_weight;
    float alpha;
    float max_delta_step;
    uint32_t max_depth;
    uint32_t max_leaves;
    uint32_t max_cat_to_onehot;
    uint32_t max_cat_threshold;
    int32_t grow_policy;        /* 0 depthwise, 1 lossguide */
    const int8_t* monotone;     /* n_features entries or NULL */
} fbgpu_tree_params;

/* A grown tree (model/tree.rs:52-79 Node, arrays by node id).  The caller
 * provides arrays of `capacity` entries (2^(max_depth+1) - 1 suffices);
 * `bin` is the right-boundary bin of a numeric split (split.rs:17-52) and
 * cats holds cat_words words (the right-going category set, a bit per code)
 * per node: at least fbgpu_ctx_cat_words(ctx), which is 8 unless a
 * categorical feature has more than 256 codes (0 is read as 8). */
typedef struct fbgpu_tree_out {
    uint32_t capacity;
    uint32_t n_nodes;
    int32_t* left;
    int32_t* right;
    uint32_t* feat;
    uint32_t* bin;
    float* gain;
    float* leaf;
    float* hess;
    uint32_t* flags;            /* bit0 leaf, bit1 default_left, bit2 categorical */
    uint32_t* cats;             /* cat_words words per node, may be NULL */
    uint32_t cat_words;
    uint32_t reserved;
} fbgpu_tree_out;

/* Result of one node's split search (split.rs:17-52 SplitCandidate;
 * backend/cuda/histogram.cu:6-11 SplitPacket).  cats: the first 8 words of
 * a categorical split's right-going set (codes < 256); fbgpu_split_cats
 * returns the whole set. */
typedef struct fbgpu_split {
    uint32_t found;
    uint32_t feat;
    uint32_t bin;
    uint32_t missing_left;
    float gain;
    uint32_t categorical;
    int64_t left_grad, left_hess, right_grad, right_hess;
    uint32_t cats[8];
} fbgpu_split;

const char* fbgpu_last_error(const fbgpu_ctx* ctx);
int32_t fbgpu_device_count(void);

/* Number of kernels this library has launched in this process (all devices
 * and threads; library kernels such as NCCL's are not counted).  A
 * diagnostic with no counterpart in the reference. */
uint64_t fbgpu_launch_count(void);

/* ---------------------------------------------------------- training context */

/* Replaces GpuTrainCtx::new_with_shape (src/backend/mod.rs:245-255). */
fbgpu_status fbgpu_ctx_create(const fbgpu_config* cfg, fbgpu_ctx** out);
void fbgpu_ctx_destroy(fbgpu_ctx* ctx);

/* ------------------------------------------------------------ row sharding */

/* Size of an NCCL unique id (NCCL_UNIQUE_ID_BYTES). */
#define FBGPU_NCCL_ID_BYTES 128

/* Creates an NCCL unique id on the calling rank (rank 0 makes one and sends
 * its bytes to the other ranks by the caller's own means).  No counterpart in
 * the reference, whose communication trait has only the single-process
 * `Local` implementation (src/training/comm.rs:10-41); this replaces that
 * trait for row sharding. */
fbgpu_status fbgpu_nccl_unique_id(uint8_t* out_id);

/* Joins `ctx` to a communicator of `nranks` contexts, one per GPU and
 * process, each holding a contiguous row range (fbgpu_config.row_offset,
 * n_rows_global).  Collectives then run on the context's stream: the max of
 * the gradient bounds and the sum of the root gradient per round, the sum of
 * the accumulated node histograms and of the per-node left counts per level.
 * Every rank must make the same calls in the same order.  Waits on the
 * communicator poll for at most `timeout_ms` (0 = 120000); past that the
 * communicator is aborted and calls return FBGPU_ETIMEOUT, later ones
 * FBGPU_ENCCL.  nranks == 1 is a no-op. */
fbgpu_status fbgpu_ctx_set_comm(fbgpu_ctx* ctx, const uint8_t* unique_id, int32_t nranks, int32_t rank,
                                uint32_t timeout_ms);

/* The same communicator, started ahead of the context: the non-blocking
 * NCCL initialization and a warm-up of two all-reduces (16 B and 8 MiB, which
 * set up NCCL's connections) run on a background host thread while the
 * caller sketches and bins its data; fbgpu_ctx_adopt_comm joins it to a
 * context (waiting for it if needed) and fbgpu_comm_free releases the
 * handle.  Every rank calls fbgpu_comm_begin, with the same unique id.  The
 * handle and the contexts that joined it share the communicator, which ends
 * when the last of them is released, so a process can keep one handle and
 * join it to the contexts of successive trainings (every rank the same
 * ones, one context at a time).  No counterpart in the reference. */
typedef struct fbgpu_comm fbgpu_comm;
fbgpu_status fbgpu_comm_begin(const uint8_t* unique_id, int32_t nranks, int32_t rank, int32_t device,
                              uint32_t timeout_ms, fbgpu_comm** out);
fbgpu_status fbgpu_ctx_adopt_comm(fbgpu_ctx* ctx, fbgpu_comm* comm);
void fbgpu_comm_free(fbgpu_comm* comm);
/* 1 when the communicator started without error, has not failed or been
 * aborted, and no live context holds it (it may join a new one); else 0. */
int32_t fbgpu_comm_usable(fbgpu_comm* comm);
/* Aborts the communicator now, without waiting for the peers (exit paths;
 * nothing may be in flight on it).  Contexts holding it fail their next
 * collective; the handle is still freed with fbgpu_comm_free. */
void fbgpu_comm_abort(fbgpu_comm* comm);

/* Feature metadata: bins per feature (cuts + 1), storage width in bytes
 * (bins.rs:58-66 BinWidth::for_feature) and categorical flags (may be NULL).
 * One-byte bins hold up to 255 bins with 255 as the missing value, or
 * exactly 256 bins for a feature that holds no missing value (every byte
 * value is a bin; the reference would store such a feature in two bytes).
 * Replaces the cuts half of GpuTrainCtx::block_session_bins
 * (src/backend/mod.rs:352-362). */
fbgpu_status fbgpu_set_features(fbgpu_ctx* ctx, const uint32_t* n_bins, const uint8_t* width,
                                const uint8_t* categorical);

/* Upload one column block (reference ColumnBlock BinData, column-major) into
 * the resident device layout.  Replaces block_session_bins /
 * block_session_resident_width (src/backend/mod.rs:352-383). */
fbgpu_status fbgpu_upload_block(fbgpu_ctx* ctx, const uint32_t* feat_ids, uint32_t n_feats, uint32_t width,
                                const void* data);

/* Labels, optional sample weights (NULL) and starting margins (per-row
 * base_margin rows, or NULL for the scalar base_margin).  Replaces
 * GpuTrainCtx::init_fast_math (src/training/mod.rs:1837-1860); in exact mode
 * the device copy of the margins is kept as well. */
fbgpu_status fbgpu_set_labels(fbgpu_ctx* ctx, const float* labels, const float* weights,
                              const float* base_margin_rows, float base_margin);

/* Exact-mode round start from host f32 gradient pairs: row-sampling mask,
 * bound scan, power-of-two scales (types.rs:366-385), fixed-point conversion
 * and root sum on the device.  Replaces upload_and_quantize_gpair_sampled
 * (src/backend/mod.rs:298-306).  sub_threshold = UINT64_MAX keeps all rows. */
fbgpu_status fbgpu_upload_and_quantize_gpair(fbgpu_ctx* ctx, const float* gpair, uint64_t sub_threshold,
                                             uint64_t seed, uint64_t tree, double* scales_out,
                                             int64_t* root_sum_out);

/* Exact-mode round start from host-quantized pairs.  Replaces upload_gpair
 * (src/backend/mod.rs:286). */
fbgpu_status fbgpu_upload_gpair(fbgpu_ctx* ctx, const int64_t* fixed, const double* scales,
                                const int64_t* root_sum);

/* Exact logistic round start: `host_exp` holds glibc expf(-margin) per row
 * (the only non-IEEE-basic step of the gradient, computed on the host like the
 * reference's exact mode, objective.rs:37-39); the device recomputes the
 * gradient from it in the host's f32 operation order and quantizes with the
 * host's scales.  No counterpart with this exact signature in the reference:
 * it is the exact-mode boundary of upload_and_quantize_gpair_sampled with
 * 4 bytes per row instead of 8. */
fbgpu_status fbgpu_round_from_exp(fbgpu_ctx* ctx, int32_t objective, const float* host_exp,
                                  uint64_t sub_threshold, uint64_t seed, uint64_t tree, const double* scales);

/* Round start with the gradient computed on the device from the resident
 * margins.  fast = 1 is gpu_math="fast" (replaces fast_gradient_and_quantize,
 * src/backend/mod.rs:220-228): no host synchronisation, the power-of-two
 * scales taken on the device, and exp evaluated in f64 and rounded once to
 * f32 (within one unit in the last place of the host expf, equal on all but
 * about 0.004 % of the inputs; the reference's fast mode uses CUDA's expf,
 * which differs on about 7 %); fast = 0 is exact
 * mode with the scales taken by the host's libm: squared error is pure f32
 * arithmetic, logistic uses the device reproduction of the host expf
 * (fbgpu_exact_exp_available must be 1).
 * scales_out / root_sum_out may be NULL (no host synchronisation then). */
fbgpu_status fbgpu_round_device(fbgpu_ctx* ctx, int32_t objective, int32_t fast, uint64_t sub_threshold,
                                uint64_t seed, uint64_t tree, double* scales_out, int64_t* root_sum_out);

/* Multiclass (multi:softprob / multi:softmax, src/training/mod.rs:2564-2800).
 * fbgpu_set_outputs makes the margins K columns (class-major), column k
 * starting at class_margins[k]; replaces init_fast_math with K margins
 * (src/backend/mod.rs:161-168).  fbgpu_multiclass_gradients computes the
 * softmax gradients of all K classes from the current margins
 * (objective.rs:1175-1219; fast = 0: the host expf reproduced on the device,
 * fbgpu_exact_exp_available must be 1); replaces fast_multiclass_begin_round
 * (mod.rs:192-194).  fbgpu_quantize_class masks, bounds and quantizes class
 * k's column for the tree with index `tree` (round * K + k) and leaves the
 * fixed gradients, root sum and scales on the device (scales by the host
 * libm, or on the device when fast; scales_out / root_sum_out may be NULL);
 * replaces fast_multiclass_gradient_and_quantize (mod.rs:195-203).
 * fbgpu_set_output_column selects the column the next fbgpu_build_tree adds
 * its leaf values to; with it, fast_multiclass_apply_delta (mod.rs:204-206)
 * has no separate step.  fbgpu_download_margins then returns K x n. */
fbgpu_status fbgpu_set_outputs(fbgpu_ctx* ctx, uint32_t n_classes, const float* class_margins);
fbgpu_status fbgpu_multiclass_gradients(fbgpu_ctx* ctx, int32_t fast);
fbgpu_status fbgpu_quantize_class(fbgpu_ctx* ctx, uint32_t cls, uint64_t sub_threshold, uint64_t seed, uint64_t tree,
                                  int32_t fast, double* scales_out, int64_t* root_sum_out);
fbgpu_status fbgpu_set_output_column(fbgpu_ctx* ctx, uint32_t cls);

/* Grow one tree on the device and add its leaf values to the resident
 * margins.  `enabled` marks the features of this tree (colsample_bytree,
 * colsample.rs:74-95), NULL = all.  Replaces the per-level loop of
 * build_tree over GpuBlockSession / GpuPartitionSession
 * (src/training/mod.rs:3569-4564): histogram_device_batch, split_cached_batch,
 * partition_resident_batch, resolve_partitions, assign_leaf_values. */
fbgpu_status fbgpu_build_tree(fbgpu_ctx* ctx, const fbgpu_tree_params* tp, const uint8_t* enabled,
                              fbgpu_tree_out* out);

/* Copy the resident margins to the host.  Replaces download_prediction_delta
 * / with_prediction_delta (src/backend/mod.rs:331-340): the device adds each
 * tree's leaf values itself, so the host receives margins instead of deltas. */
fbgpu_status fbgpu_download_margins(fbgpu_ctx* ctx, float* out);

/* Whether exact-mode logistic gradients can be computed on the device: the
 * host C library's expf (which Rust's f32::exp calls in the reference,
 * objective.rs:37-39) is reproduced on the device by an f64 exp plus a table
 * of the inputs where the two differ, and the table has been checked against
 * this host's expf.  Returns 1 or 0; *why gets the reason when 0.  No
 * counterpart in the reference, whose exact mode always computes gradients on
 * the host. */
int32_t fbgpu_exact_exp_available(const char** why);

/* Compares the device's reproduction of the host expf with the host's own
 * expf on the inputs with bit patterns [begin, begin + count) and stores the
 * number of differing results; `report` (16 words or NULL) receives up to four
 * (input, host expf, device result, host fexp_core) bit quadruples (test entry
 * point; allocates device memory). */
fbgpu_status fbgpu_expf_check(int32_t device, uint32_t begin, uint32_t count, uint64_t* mismatches,
                              uint32_t* report);

/* ---------------------------------------------------------- component calls */

/* Histogram of `rows` (host array, ascending or not; NULL = every row) over
 * all features, with the context's current fixed-point gradients or `fixed`
 * (host, 2 x n_rows int64) when given.  out: total_bins x 2 int64.  The C
 * form of hist::build (src/training/hist.rs:35-62) and of
 * GpuBlockSession::histogram_device_batch (src/backend/mod.rs:433-439). */
fbgpu_status fbgpu_histogram(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n_sel, const int64_t* fixed,
                             int64_t* out);

/* Best split of one node from a host histogram.  The C form of
 * split::best_split_in_block_typed (src/training/split.rs:331-461) as the
 * device split kernels compute it. */
fbgpu_status fbgpu_eval_split(fbgpu_ctx* ctx, const int64_t* hist, const int64_t* node_sum, const double* scales,
                              const fbgpu_tree_params* tp, float lower, float upper, const uint8_t* enabled,
                              fbgpu_split* out);

/* Stable partition of `rows` by one split: left rows first, then right.
 * Replaces GpuPartitionSession::partition / partition_categorical
 * (src/backend/mod.rs:468-483). cats: 8 words or NULL. */
fbgpu_status fbgpu_partition(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n, uint32_t feat, uint32_t bin,
                             int32_t missing_left, const uint32_t* cats, uint32_t* out_rows, uint64_t* n_left);

/* fbgpu_partition by a category set of any width: n_words words, a bit per
 * code (codes beyond them go left).  Replaces
 * GpuPartitionSession::partition_categorical (src/backend/mod.rs:476-483)
 * for features of up to 65534 codes (src/data/categorical.rs:19-28). */
fbgpu_status fbgpu_partition_set(fbgpu_ctx* ctx, const uint32_t* rows, uint64_t n, uint32_t feat,
                                 int32_t missing_left, const uint32_t* cats, uint32_t n_words, uint32_t* out_rows,
                                 uint64_t* n_left);

/* Words of a category set in this context: 8, or ceil(bins / 32) of its
 * widest categorical feature (fbgpu_tree_out.cat_words must be at least
 * this).  No counterpart in the reference, whose bitsets are Vec<u32>. */
uint32_t fbgpu_ctx_cat_words(const fbgpu_ctx* ctx);

/* The whole right-going category set of the last fbgpu_eval_split (n_words
 * words; FBGPU_EINPUT if the set does not fit).  Completes fbgpu_split.cats
 * for features of more than 256 codes. */
fbgpu_status fbgpu_split_cats(fbgpu_ctx* ctx, uint32_t* out, uint32_t n_words);

/* Stable partition of device row ids by one numeric or categorical split,
 * allocating no device memory.  No counterpart in the reference: it exists for
 * callers that own every device allocation themselves and cannot call
 * cudaMalloc (the reference's Rust host keeps all allocation on its side,
 * src/backend/mod.rs:7-10).  All pointers are device pointers except `cats`
 * (8 host words, the right-going categories < 256, or NULL for a numeric
 * split `bin < split bin goes left`).  `bins` is a row-major record matrix:
 * the feature's bin of row r is the `width`-byte value at
 * bins + r*stride + byte_off, and a row whose bin equals `missing_bin` is
 * missing (the reference's layout: 255 for one byte, 65535 for two bytes;
 * 0xFFFFFFFF for a feature that holds no missing value, such as a 256-bin
 * feature stored in one byte).  For two-byte bins the records' address,
 * stride and byte_off must be even; rows, out_rows and n_left 4-byte aligned;
 * rows and out_rows must not overlap (no in-place partition).  Writes the left
 * rows then the right rows of `rows` to `out_rows` in input order, and the
 * left count to *n_left.  Work is enqueued on `stream` (a cudaStream_t of the
 * current device, NULL = default stream).  The kernels' scratch is one fixed
 * 512 KiB static device array per device, so at most 268435456 rows per call
 * (larger requests, like every rule above, fail with FBGPU_EINPUT).  The
 * first call on a device looks the array up (cudaGetSymbolAddress), and again
 * the first call after the device's context was replaced (cudaDeviceReset);
 * make those calls before any stream capture.  Every call shares the array:
 * calls that overlap on the GPU race. */
fbgpu_status fbgpu_partition_noalloc(const void* bins, uint32_t stride, uint32_t width, uint32_t byte_off,
                                     uint32_t missing_bin, const uint32_t* rows, uint64_t n, uint32_t bin,
                                     int32_t missing_left, const uint32_t* cats, uint32_t* out_rows,
                                     uint32_t* n_left, void* stream);

/* Updates per second of the exact histogram update alone (no reference
 * counterpart: a measurement of this engine's shared-memory atomic ceiling).
 * Every (row, feature) update adds a gradient pair as two 64-bit sums modulo
 * 2^64 to a 256-bin shared histogram, with rows generated in registers, on
 * every SM of `device`; scheme 0 is the histogram kernel's (returning
 * low-word atomic, carry into the high word), 1 the same with the low-word
 * atomics of 4 updates issued first, 2 native 64-bit shared atomics, 3 four
 * non-returning 32-bit atomics (not exact: the pipe's ceiling).  iters:
 * updates per thread, a multiple of 8. */
fbgpu_status fbgpu_hist_atomic_ceiling(int32_t device, int32_t scheme, uint32_t iters, double* updates_per_s);

/* The power-of-two quantizer scale of each bound `max_abs[i]` (the largest
 * |gradient| or |Hessian| of a round, an f32 value) for `n_rows` rows, as
 * exact-mode training computes it on the device: the reference's pow2_scale
 * (src/types.rs:366-385, 2^floor(log2((2^62 / n_rows) / max_abs)) with the
 * host's log2, clamped to 2^-1000..2^1000, 1.0 when that is not a positive
 * finite number).  device >= 0 evaluates on that GPU, device < 0 on the host;
 * both use the same code.  No reference counterpart as an entry point: the
 * reference computes this on the host inside each round. */
fbgpu_status fbgpu_quantizer_scales(int32_t device, const float* max_abs, uint64_t count, uint64_t n_rows,
                                    double* out);
/* Sum modulo 2^64 of mix(b, scale(f32 with bits b)) over b in [lo_bits,
 * hi_bits), host, all cores: compared with the same digest of the
 * reference's pow2_scale over every positive f32 (tests).  mix is the
 * SplitMix64 finalizer of (scale bits) ^ (b * 0x9E3779B97F4A7C15). */
uint64_t fbgpu_quantizer_scale_digest(uint32_t lo_bits, uint32_t hi_bits, uint64_t n_rows);

/* ---------------------------------------------------------- explanation models */

/* A model for device prediction and SHAP.  Node arrays of all trees back to
 * back; tree t owns nodes [tree_off[t], tree_off[t+1]) with tree-local child
 * indices; value = leaf value (leaf) or split condition (numeric split);
 * flags: bit0 leaf, bit1 default_left, bit2 categorical; categorical node i
 * tests cat_words[cat_off[i] .. cat_off[i] + cat_len[i]).  Replaces
 * GpuExplainModel::new and GpuInferenceModel construction
 * (src/backend/cuda/explain.rs:355, src/backend/cuda/inference.rs:67). */
fbgpu_status fbgpu_model_create(int32_t device, uint32_t n_features, uint32_t n_trees, const uint32_t* tree_off,
                                const int32_t* left, const int32_t* right, const uint32_t* feat, const float* value,
                                const uint8_t* flags, const float* hess, const uint32_t* cat_off,
                                const uint32_t* cat_len, const uint32_t* cat_words, uint64_t n_cat_words,
                                float base_margin, fbgpu_model** out);
void fbgpu_model_destroy(fbgpu_model* m);

/* Raw margins of host rows (row-major n x n_features).  Replaces
 * GpuInferenceModel::predict_margins (src/backend/cuda/inference.rs:300-339). */
fbgpu_status fbgpu_predict(fbgpu_model* m, const float* X, uint64_t n, float* out);
/* The same on device buffers, enqueued on `stream` (a cudaStream_t). */
fbgpu_status fbgpu_predict_device(fbgpu_model* m, const float* X, uint64_t n, float* out, void* stream);

/* QuadratureTreeSHAP contributions, n x (n_features + 1), bias last.
 * Replaces GpuExplainModel::compute (src/backend/cuda/explain.rs:491). */
fbgpu_status fbgpu_shap(fbgpu_model* m, const float* X, uint64_t n, float* out);
fbgpu_status fbgpu_shap_device(fbgpu_model* m, const float* X, uint64_t n, float* out, void* stream);

/* The other explanation kinds of GpuExplainModel::compute
 * (src/backend/cuda/explain.rs:491; src/model/explain.rs Kind):
 *   FBGPU_EXPLAIN_LEAF          n x n_trees: the node index each tree's traversal ends at (as float);
 *   FBGPU_EXPLAIN_APPROX        n x (n_features + 1): Saabas contributions (approx_contribs), bias last;
 *   FBGPU_EXPLAIN_INTERACTIONS  n x (n_features + 1)^2: SHAP interaction values, bias row/column last. */
#define FBGPU_EXPLAIN_LEAF 0
#define FBGPU_EXPLAIN_APPROX 1
#define FBGPU_EXPLAIN_INTERACTIONS 2
fbgpu_status fbgpu_explain(fbgpu_model* m, int32_t kind, const float* X, uint64_t n, float* out);
fbgpu_status fbgpu_explain_device(fbgpu_model* m, int32_t kind, const float* X, uint64_t n, float* out,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif
