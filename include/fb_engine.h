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
    int32_t objective;          /* 0 reg:squarederror, 1 binary:logistic, 2 multi:softprob, 3 multi:softmax */
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
    uint32_t num_class;         /* multi:softprob / multi:softmax: classes, >= 2 (K trees per round) */
    const float* class_margins; /* multiclass: the K base margins over all rows, or NULL (estimated from the
                                   booster's labels, or base_score K times); a row-sharded multiclass
                                   booster needs them or base_score (fb_class_margins on all labels) */
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
/* The dataset of fb_dataset_from_dense (cuts == NULL) or fb_dataset_with_cuts
 * (cuts and F+1 offsets given), quantized on CUDA device `device`: the rows
 * are copied to the device once, the weighted quantile sketch runs there
 * (cuts bit-identical to fb_dataset_from_dense; with weights, or max_bin >
 * 1024, the host sketch supplies them), and the bins are written straight
 * into the row records a booster on that device trains from, which stay
 * resident (no host copy of the bins exists).  A booster built from it must
 * use the same device.  Replaces the sketch + quantize_row_major passes of
 * DenseSource::new_weighted_with_nthread (src/source/dense.rs:99-209,
 * src/data/sketch.rs:128-302) for device training. */
fb_dataset* fb_dataset_on_device(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* weights,
                                 const uint8_t* categorical, const float* cuts, const uint32_t* offsets,
                                 int32_t nthread, int32_t device);
/* fb_dataset_on_device with the features given column-major: X holds F
 * columns of n values back to back (feature f at X + f * n), the layout a
 * columnar file (Parquet / Arrow) decodes into; same sketch, bins and errors.
 * Replaces the column-chunk ingest of src/source/parquet_source.rs:541-620
 * (open / open_with_cuts) after the reader has decoded the feature columns. */
fb_dataset* fb_dataset_on_device_columns(const float* X, uint64_t n, uint32_t F, uint32_t max_bin,
                                         const float* weights, const uint8_t* categorical, const float* cuts,
                                         const uint32_t* offsets, int32_t nthread, int32_t device);
/* Device holding the dataset's bins, or -1 for a host dataset. */
int32_t fb_dataset_device(const fb_dataset* d);
/* Cuts of the listed features only, with the sketch of fb_dataset_from_dense
 * (features are sketched independently, so the ranks of a row-sharded run
 * can split the features between them and exchange the cuts).  The cuts of
 * feats[i] are written back to back into `cuts`, their count into counts[i].
 * Returns the total, or -1 (fb_last_error) when it exceeds `cap` or an input
 * is invalid.  Replaces the per-feature part of DenseSource::new_weighted
 * (src/source/dense.rs:136-209, sketch.rs:128-302). */
int64_t fb_sketch_features(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* weights,
                           const uint8_t* categorical, const uint32_t* feats, uint32_t n_feats, int32_t nthread,
                           float* cuts, uint32_t* counts, uint64_t cap);
/* fb_sketch_features computed on CUDA device `device` (the rows are copied
 * there once, copied by nthread host threads, 0 = the OpenMP default); the
 * same cuts, bit for bit.  With weights, or max_bin > 1024, the host sketch
 * runs instead. */
int64_t fb_sketch_features_device(const float* X, uint64_t n, uint32_t F, uint32_t max_bin, const float* weights,
                                  const uint8_t* categorical, const uint32_t* feats, uint32_t n_feats, int32_t nthread,
                                  int32_t device, float* cuts, uint32_t* counts, uint64_t cap);
/* The base_score estimated from the labels when none is given: the label mean
 * (weighted when weights != NULL), summed in f64 in row order
 * (src/objective.rs:41-61). */
float fb_label_mean(const float* labels, const float* weights, uint64_t n);
/* The unweighted label mean's f64 accumulator before its rounding to f32
 * (objective.rs:41-61: acc = acc + label / n in row order), the value
 * fb_label_mean rounds.  Exposed so that its exactness against the row loop
 * can be checked at f64. */
double fb_label_mean_f64(const float* labels, uint64_t n);
/* The base score a booster takes when base_score is not given (objective.rs:
 * 403-493 initial_base_score; objective 0 squared error, 1 logistic): the
 * label mean, or with |scale_pos_weight - 1| > 1e-6 one Newton step from
 * margin 0 over the gradient weights (weights may be NULL). */
float fb_initial_base_score(int32_t objective, const float* labels, const float* weights, uint64_t n,
                            float scale_pos_weight);
/* The multiclass base margins (objective.rs:1225-1247 initial_class_margins):
 * weighted class counts summed in f32 in row order, log(count / sum_w + 1e-6),
 * minus their mean; K values to out.  Labels must be integers in [0, K). */
int32_t fb_class_margins(const float* labels, const float* weights, uint64_t n, uint32_t K, float* out);
void fb_dataset_free(fb_dataset* d);
uint64_t fb_dataset_rows(const fb_dataset* d);
/* Cuts: copies up to cap values; returns the total.  offsets: F+1 entries. */
int64_t fb_dataset_cuts(const fb_dataset* d, float* cuts, uint32_t* offsets, uint64_t cap);
/* Column-major bins of feature f (n entries, missing = 255 / 65535). */
int32_t fb_dataset_column(const fb_dataset* d, uint32_t f, uint16_t* out);

/* A booster trains every row of the dataset on one device (p->device).  It
 * allocates all device memory at creation and none during training. */
fb_booster* fb_booster_create(const fb_dataset* d, const float* labels, const float* weights, const fb_params* p);
/* A booster over one row shard of a run on `nranks` GPUs, one process per
 * GPU: the dataset holds rows [row_offset, row_offset + rows) of
 * n_rows_global, binned with the cuts of the whole data; labels and weights
 * are those rows'.  p->base_score must be set (fb_label_mean of all labels).
 * Every rank passes the same parameters and the same NCCL unique id
 * (fbgpu_nccl_unique_id on rank 0) and calls update with the same counts; each
 * then holds the same model, byte for byte the single-GPU model in exact
 * mode.  Collective waits give up after timeout_ms (0 = 120000).  No
 * counterpart in the reference (single GPU only). */
fb_booster* fb_booster_create_sharded(const fb_dataset* shard, const float* labels, const float* weights,
                                      const fb_params* p, uint64_t row_offset, uint64_t n_rows_global,
                                      const uint8_t* nccl_id, int32_t nranks, int32_t rank, uint32_t timeout_ms);
/* fb_booster_create_sharded with a communicator already started by
 * fbgpu_comm_begin (include/fbgpu.h), so its initialization overlapped the
 * data preparation, or kept from an earlier training; the booster shares
 * the communicator with the handle (which is still freed with
 * fbgpu_comm_free). */
struct fbgpu_comm;
fb_booster* fb_booster_create_sharded_comm(const fb_dataset* shard, const float* labels, const float* weights,
                                           const fb_params* p, uint64_t row_offset, uint64_t n_rows_global,
                                           struct fbgpu_comm* comm, int32_t nranks, int32_t rank);
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
/* Of the histogram device ms above: the device ms of the per-level histogram
 * all-reduces of a row-sharded booster (0 on one GPU), while statistics are
 * on.  No counterpart in the reference (it has no multi-GPU path). */
double fb_booster_collective_ms(const fb_booster* b);
/* The (row, feature) updates the histogram kernels made while statistics
 * were on: accumulated rows x enabled features, summed over the levels (no
 * reference counterpart; the histogram's work in the unit of
 * fbgpu_hist_atomic_ceiling). */
double fb_booster_hist_updates(const fb_booster* b);
void fb_booster_set_stats(fb_booster* b, int32_t on);
fb_model* fb_booster_model(fb_booster* b);
/* Current training margins of the booster's rows (host copy). */
int32_t fb_booster_margins(fb_booster* b, float* out);

/* One-call training: dataset + booster + n_rounds (the reference's train). */
fb_model* fb_train(const float* X, uint64_t n, uint32_t F, const float* y, const float* w, const uint8_t* categorical,
                   const fb_params* p, uint32_t n_rounds);

/* A model from flat tree arrays, as the reference's Model::load_model parses
 * an XGBoost-compatible JSON (src/model/tree.rs:760-960): trees back to back,
 * tree t owning nodes [tree_off[t], tree_off[t+1]) with tree-local children
 * (left < 0: a leaf, whose value is leaf[i]); a split's condition is cond[i]
 * and its default direction default_left[i]; a categorical split (is_cat[i])
 * sends the categories of its bitset cat_words[cat_off[i] .. + cat_len[i]]
 * right (n_cat_words words in all).  objective: 0 reg:squarederror, 1
 * binary:logistic, 2 multi:softprob, 3 multi:softmax (num_class >= 2 and K
 * class_margins; tree t belongs to class t % K).  feature_types may be NULL
 * (all numeric).  Returns NULL with fb_last_error on an inconsistent model:
 * besides ranges, every tree must be a tree (tree.rs:1363-1447): a node has
 * both children or none, each node at most one parent, the root none, and
 * every node is reached from the root exactly once. */
fb_model* fb_model_create(uint32_t n_features, int32_t objective, float base_score, float scale_pos_weight,
                          uint32_t num_class, const float* class_margins, const uint8_t* feature_types,
                          uint32_t n_trees, const uint32_t* tree_off, const int32_t* left, const int32_t* right,
                          const uint32_t* feat, const float* cond, const uint8_t* default_left, const float* leaf,
                          const float* gain, const float* hess, const uint8_t* is_cat, const uint32_t* cat_off,
                          const uint32_t* cat_len, const uint32_t* cat_words, uint64_t n_cat_words);
void fb_model_free(fb_model* m);
uint32_t fb_model_num_trees(const fb_model* m);
uint32_t fb_model_num_features(const fb_model* m);
float fb_model_base_margin(const fb_model* m);
int64_t fb_model_json(const fb_model* m, char* buf, int64_t cap);
/* Flat arrays of tree t (node count returned; any array may be NULL).  cats
 * receives 8 words per node (the right-going category set). */
int64_t fb_model_tree(const fb_model* m, uint32_t t, int32_t* left, int32_t* right, uint32_t* feat, float* cond,
                      uint8_t* default_left, float* leaf, uint8_t* is_leaf, float* gain, float* hess, uint32_t* cats);
/* The right-going category set of node `node` of tree t: returns its length
 * in 32-bit words (0 for a numeric split or a leaf, -1 for a bad index) and
 * copies at most cap words to out.  fb_model_tree's cats holds only the
 * first 8 words (codes < 256). */
int64_t fb_model_node_cats(const fb_model* m, uint32_t t, uint32_t node, uint32_t* out, uint32_t cap);
/* Raw margins of host rows, computed on the device: n values, or n x K
 * (row-major) for a multiclass model of K outputs (src/model/tree.rs:468-480
 * predict_margins_upto). */
int32_t fb_model_predict(fb_model* m, const float* X, uint64_t n, float* out, int32_t device);
/* Outputs per row: num_class for multi:softprob / multi:softmax, else 1. */
uint32_t fb_model_num_outputs(const fb_model* m);
/* Multiclass prediction transform of n x K margins (objective.rs:1260-1333
 * transform_rows): multi:softprob turns each row into probabilities in
 * place; multi:softmax writes each row's class index (first maximum) to
 * classes[r]. */
int32_t fb_model_transform(const fb_model* m, float* margins, uint64_t n, float* classes);
/* The model's device copy on `device` as an include/fbgpu.h handle (owned by
 * the model, valid until the model is freed or gains trees), for
 * fbgpu_predict_device / fbgpu_shap_device on device-resident rows.  For a
 * multiclass model the handle holds all trees in order with a zero base margin
 * (what fbgpu_explain's leaf indices need); per-class margins and SHAP groups
 * come from fb_model_predict / fb_model_shap. */
struct fbgpu_model* fb_model_device(fb_model* m, int32_t device);
/* SHAP contributions n x (F+1) on the device; n x K x (F+1) for a
 * multiclass model (one group per class, src/model/explain.rs:704-727). */
int32_t fb_model_shap(fb_model* m, const float* X, uint64_t n, float* out, int32_t device);
/* Leaf indices (kind 0, n x n_trees), Saabas contributions (kind 1,
 * n x (F+1)) or SHAP interaction values (kind 2, n x (F+1)^2) on the device;
 * kinds 1 and 2 of a multiclass model carry a class axis after the row
 * (the reference's predict(pred_leaf / approx_contribs / pred_interactions),
 * src/model/explain.rs Kind). */
int32_t fb_model_explain(fb_model* m, int32_t kind, const float* X, uint64_t n, float* out, int32_t device);

#ifdef __cplusplus
}
#endif
#endif
