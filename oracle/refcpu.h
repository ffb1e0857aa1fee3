/*
 * refcpu — CPU restatement of the FerrisBoost reference engine.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the correctness oracle and the
 * timed CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it.  The product library
 * (ferrisboost_b200/libfbgpu.so) never links, loads or calls it.
 *
 * Parity is pinned against the XGBoost 3.4.1 golden margins the reference
 * ships in tests/fixtures (index.json, weighted_index.json,
 * monotone_index.json), copied into tests/golden/.  See oracle/refcpu.cpp for
 * the per-function citations of the reference sources it restates.
 */
#ifndef FB_REFCPU_H
#define FB_REFCPU_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Training parameters; field meanings follow TrainParams (src/types.rs:433-686). */
typedef struct rc_params {
    int32_t objective;          /* 0 reg:squarederror, 1 binary:logistic, 2 multi:softprob, 3 multi:softmax */
    int32_t grow_policy;        /* 0 depthwise, 1 lossguide */
    uint32_t n_rounds;
    uint32_t max_depth;
    uint32_t max_leaves;        /* 0 = unlimited */
    uint32_t max_bin;
    float eta;
    float lambda;
    float gamma;
    float min_child_weight;
    float alpha;
    float max_delta_step;
    float scale_pos_weight;
    float subsample;
    float colsample_bytree;
    float base_score;           /* NaN = estimate from labels */
    uint64_t seed;
    uint32_t max_cat_to_onehot;
    uint32_t max_cat_threshold;
    int32_t nthread;            /* 0 = all cores */
    const int8_t* monotone;     /* n_features entries or NULL */
    const uint8_t* categorical; /* n_features entries or NULL */
    uint32_t num_class;         /* multi:softprob / multi:softmax: classes (>= 2) */
} rc_params;

void rc_default_params(rc_params* p);

/* Train on a row-major float32 matrix (NaN = missing).  Returns a model
 * handle or NULL (message via rc_last_error). */
void* rc_train(const float* X, uint64_t n, uint32_t F, const float* y,
               const float* w, const rc_params* p);
const char* rc_last_error(void);
/* rc_train with rows sharded over n_ranks threads as ranks (depthwise growth;
 * lossguide trains unsharded): partial histograms per rank summed by a fake
 * collective, the accumulated child chosen by global hessian sums, and with
 * feature_sharded the split search split by feature range with the
 * winners gathered.  The models must equal rc_train's. */
void* rc_train_sharded(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const rc_params* p,
                       int32_t n_ranks, int32_t feature_sharded);
/* Wall seconds of the last rc_train on this thread: setup (sketch, bins) and
 * each round.  Returns the number of rounds. */
int32_t rc_last_timing(double* setup_s, double* round_s, int32_t cap);
void rc_model_free(void* model);
uint32_t rc_model_num_trees(void* model);
/* XGBoost-compatible JSON; returns the length (writes at most cap bytes). */
int64_t rc_model_json(void* model, char* buf, int64_t cap);
/* objective.rs:1175-1219 softmax gradients: margins K x n (class-major) ->
 * out K x n (g, h) pairs; w may be NULL. */
void rc_softmax_gradients(const float* margins, const float* y, const float* w, uint64_t n, uint32_t K, float* out);
/* objective.rs:1225-1247 initial_class_margins. */
void rc_class_margins(const float* y, const float* w, uint64_t n, uint32_t K, float* out);
/* Outputs per row: num_class for a multiclass model, else 1. */
uint32_t rc_model_num_outputs(void* model);
/* Flat tree arrays of tree t (node count returned; arrays may be NULL). */
int64_t rc_model_tree(void* model, uint32_t t, uint32_t* feat, float* cond,
                      int32_t* left, int32_t* right, uint8_t* default_left,
                      float* leaf, uint8_t* is_leaf, float* gain, float* hess);
float rc_model_base_margin(void* model);
/* A model from the flat arrays of an XGBoost JSON document (parsed by the
 * caller; model/tree.rs:760-960 is the reference's loader).  Tree t holds
 * nodes [tree_off[t], tree_off[t+1]); a node with left < 0 is a leaf whose
 * value is value[i], otherwise value[i] is its threshold.  Node i's
 * right-going category codes are cats[cat_off[i] .. cat_off[i] + cat_len[i]]
 * (cat_len 0: a numeric split).  class_margins holds num_class base margins
 * for a multiclass model (else NULL).  feature_types: n_features flags
 * (1 = categorical) or NULL.  Returns NULL with rc_last_error on bad input. */
void* rc_model_load(uint32_t n_trees, const uint32_t* tree_off, const int32_t* left, const int32_t* right,
                    const uint32_t* feat, const float* value, const uint8_t* default_left, const float* gain,
                    const float* hess, const uint64_t* cat_off, const uint32_t* cat_len, const uint32_t* cats,
                    uint32_t n_features, int32_t objective, float base_score, const float* class_margins,
                    uint32_t num_class, float scale_pos_weight, const uint8_t* feature_types);
void rc_predict_margin(void* model, const float* X, uint64_t n, float* out,
                       int32_t nthread);
/* QuadratureTreeSHAP contributions: n x (F+1), bias last. */
void rc_shap(void* model, const float* X, uint64_t n, float* out,
             int32_t nthread);

/* Leaf node index of every tree, n x T (as float, explain.rs:690-701). */
void rc_pred_leaf(void* model, const float* X, uint64_t n, float* out, int32_t nthread);
/* Saabas contributions (approx_contribs), n x (F+1), bias last. */
void rc_pred_approx(void* model, const float* X, uint64_t n, float* out, int32_t nthread);
/* SHAP interaction values, n x (F+1) x (F+1). */
void rc_pred_interactions(void* model, const float* X, uint64_t n, float* out, int32_t nthread);

/* ---- component entry points used by the kernel parity tests ---- */

/* Weighted quantile sketch cuts.  offsets has F+1 entries; returns the total
 * number of cuts, or -1 if cap is too small. */
int64_t rc_sketch(const float* X, uint64_t n, uint32_t F, uint32_t max_bin,
                  const float* w, const uint8_t* categorical, float* cuts,
                  uint32_t* offsets, uint64_t cap, int32_t nthread);
/* Bin codes, column-major F x n; missing = 255 for features stored at 8 bits
 * and 65535 for features stored at 16 bits. */
void rc_quantize(const float* X, uint64_t n, uint32_t F, const float* cuts,
                 const uint32_t* offsets, const uint8_t* categorical,
                 uint16_t* out);
/* Power-of-two quantizer scales (grad, hess) for n_rows rows. */
int rc_quantizer(const float* gpair, uint64_t n, uint64_t n_rows,
                 double* scales);
/* types.rs:366-385 pow2_scale of each f32 bound, and a digest of it over the
 * f32 bit patterns [lo_bits, hi_bits): the sum modulo 2^64 of the SplitMix64
 * finalizer of (scale bits) ^ (b * 0x9E3779B97F4A7C15). */
void rc_pow2_scales(const float* max_abs, uint64_t count, uint64_t n_rows, double* out);
uint64_t rc_pow2_scale_digest(uint32_t lo_bits, uint32_t hi_bits, uint64_t n_rows);
/* Fixed-point gradients round(v * scale) and their sum. */
void rc_to_fixed(const float* gpair, uint64_t n, const double* scales,
                 int64_t* out, int64_t* sum);
/* Histogram of the rows `rows` (NULL = all) over column-major bins.
 * out has feat_offsets[F] pairs and must be zeroed by the caller. */
void rc_hist(const uint16_t* bins, uint64_t n, uint32_t F,
             const uint32_t* feat_offsets, const uint16_t* missing,
             const int64_t* gpair, const uint32_t* rows, uint64_t n_sel,
             int64_t* out);
/* Best split of one node.  packet: [feat, bin, missing_left, found] as
 * uint32 plus gain (float) and left/right sums (int64 x4). */
typedef struct rc_split {
    uint32_t found;
    uint32_t feat;
    uint32_t bin;
    uint32_t missing_left;
    float gain;
    float pad;
    int64_t left_g, left_h, right_g, right_h;
    uint32_t cats[8]; /* right-going categories (codes < 256) */
} rc_split;
void rc_best_split(const int64_t* hist, uint32_t F, const uint32_t* feat_offsets,
                   const int64_t* node_sum, const double* scales,
                   const rc_params* p, float lower, float upper,
                   const uint8_t* enabled, rc_split* out);
/* colsample_bytree of one tree (data/colsample.rs:29-104): the sampled
 * feature ids, ascending, into out (nf entries of room); returns how many. */
uint32_t rc_sample_features(uint32_t nf, float rate, uint64_t seed, uint64_t round, uint32_t* out);
/* subsample of one tree (data/subsample.rs:45-78): out[r] = 1 when row r
 * keeps its gradient. */
void rc_rows_selected(uint64_t n, float rate, uint64_t seed, uint64_t tree, uint8_t* out);

#ifdef __cplusplus
}
#endif
#endif
