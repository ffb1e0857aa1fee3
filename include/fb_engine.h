/*
 * fb_engine.h — engine-level C ABI of libfbgpu.so, used by the Python
 * package (ferrisboost_b200) the way the reference's PyO3 layer uses its Rust
 * training engine (src/python/mod.rs: _core.train_dense :4179,
 * Model.predict :2667, save_model / load_model).
 *
 * The engine owns dataset preparation (weighted quantile sketch and column
 * blocks, the reference's DenseSource), the round loop (gradients, quantizer,
 * column sampling, tree assembly; src/training/mod.rs:1299-2376) and the
 * model (XGBoost-compatible JSON, src/model/tree.rs:600-1257); every
 * per-row / per-bin step runs on the device through include/fbgpu.h.
 */
#ifndef FB_ENGINE_H
#define FB_ENGINE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fb_dataset fb_dataset;
typedef struct fb_booster fb_booster;
typedef struct fb_model fb_model;

/* Training parameters (TrainParams, src/types.rs:433-686, and the objective /
 * base_score of TrainConfig, src/training/mod.rs:627-675). */
typedef struct fb_params {
    int32_t objective;          /* 0 reg:squarederror, 1 binary:logistic */
    int32_t grow_policy;        /* 0 depthwise, 1 lossguide */
    uint32_t max_depth;
    uint32_t max_leaves;
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
    float base_score;           /* NaN = estimate from the labels */
    uint64_t seed;
    uint32_t max_cat_to_onehot;
    uint32_t max_cat_threshold;
    int32_t nthread;            /* host threads, 0 = all */
    int32_t gpu_math;           /* 0 exact, 1 fast */
    int32_t device;
    const int8_t* monotone;     /* n_features or NULL */
} fb_params;

void fb_default_params(fb_params* p);
const char* fb_last_error(void);

/* Dense row-major float32 matrix (NaN = missing) -> cuts + column blocks.
 * Replaces DenseSource::new_weighted_with_nthread (src/source/dense.rs:99-209). */
fb_dataset* fb_dataset_from_dense(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* weights,
                                  const uint8_t* categorical, int32_t nthread);
/* Same, with cuts given (validation sets reuse the training cuts;
 * DenseSource::with_cuts, src/source/dense.rs:215-235). */
fb_dataset* fb_dataset_with_cuts(const float* X, uint64_t n, uint32_t F, const float* cuts, const uint32_t* offsets,
                                 const uint8_t* categorical, int32_t nthread);
void fb_dataset_free(fb_dataset* d);
uint64_t fb_dataset_rows(const fb_dataset* d);
/* Cuts: copies up to cap values; returns the total.  offsets: F+1 entries. */
int64_t fb_dataset_cuts(const fb_dataset* d, float* cuts, uint32_t* offsets, uint64_t cap);
/* Column-major bins of feature f (n entries, missing = 255 / 65535). */
int32_t fb_dataset_column(const fb_dataset* d, uint32_t f, uint16_t* out);

/* A booster trains every row of the dataset on one device (p->device).  It
 * allocates all device memory at creation and none during training. */
fb_booster* fb_booster_create(const fb_dataset* d, const float* labels, const float* weights, const fb_params* p);
void fb_booster_free(fb_booster* b);
/* Train n_rounds more trees. */
int32_t fb_booster_update(fb_booster* b, uint32_t n_rounds);
/* Timing of the last update call: [0] wall ms, [1] host-side gradient phase
 * ms, [2] host-side tree phase ms, [3] device ms between CUDA events on the
 * training stream, [4] histogram-kernel device ms, [5] histogram launches,
 * [6] histogram algorithmic bytes, [7] trees so far.  [4..6] are filled only
 * while statistics are on (fb_booster_set_stats), which adds CUDA events
 * around every histogram phase. */
void fb_booster_timing(const fb_booster* b, double* out8);
void fb_booster_set_stats(fb_booster* b, int32_t on);
fb_model* fb_booster_model(fb_booster* b);
/* Current training margins of the booster's rows (host copy). */
int32_t fb_booster_margins(fb_booster* b, float* out);

/* One-call training: dataset + booster + n_rounds (the reference's train). */
fb_model* fb_train(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const uint8_t* categorical,
                   const fb_params* p, uint32_t n_rounds);

void fb_model_free(fb_model* m);
uint32_t fb_model_num_trees(const fb_model* m);
uint32_t fb_model_num_features(const fb_model* m);
float fb_model_base_margin(const fb_model* m);
int64_t fb_model_json(const fb_model* m, char* buf, int64_t cap);
/* Flat arrays of tree t (node count returned; any array may be NULL).  cats
 * receives 8 words per node (the right-going category set). */
int64_t fb_model_tree(const fb_model* m, uint32_t t, int32_t* left, int32_t* right, uint32_t* feat, float* cond,
                      uint8_t* default_left, float* leaf, uint8_t* is_leaf, float* gain, float* hess, uint32_t* cats);
/* Raw margins of host rows, computed on the device. */
int32_t fb_model_predict(fb_model* m, const float* X, uint64_t n, float* out, int32_t device);
/* SHAP contributions n x (F+1) on the device. */
int32_t fb_model_shap(fb_model* m, const float* X, uint64_t n, float* out, int32_t device);

#ifdef __cplusplus
}
#endif
#endif
