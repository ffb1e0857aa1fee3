// Device-side tree growth for sm_100a.
//
// One tree is grown level by level entirely on the device: the histogram,
// split, decision, partition and next-level kernels of every level are
// enqueued back to back on one stream and read their node counts from device
// memory (TreeState), so growing a tree needs no host round trip.  The host
// reads the finished tree arrays once.  Kernels launched with an upper-bound
// grid return early for the nodes / chunks that do not exist in a level.
//
// The arithmetic restates the reference CPU engine (mdai001/FerrisBoost):
// histograms are i64 fixed-point sums modulo 2^64 (src/training/hist.rs),
// split scoring follows src/training/split.rs:182-461 in the given-weight
// form, partitions are stable (src/training/mod.rs:5169-5429) and leaf values
// follow src/training/mod.rs:5069-5103.
#pragma once
#include "common.cuh"
#include "fexp.h"
#include "qscale.h"

namespace fbg {

constexpr int kSplitThreads = 256;
constexpr int kMaxBinsPerThread = 4;  // features up to 1024 bins per CTA scan
constexpr uint32_t kChunkRows = 4096; // partition / leaf chunk
constexpr int kPartThreads = 512;
constexpr int kPartItems = kChunkRows / kPartThreads;
constexpr uint32_t kWalkNodes = 512;  // k_tree_walk keeps trees of up to this many nodes in shared memory
constexpr int kHistThreads = 512;
constexpr int kHistLpfThreads = 1024;

// A histogram tile: a set of features of one storage block whose bins fit in
// shared memory.  Features are listed in TileFeat[feat_begin, feat_begin+n).
struct TileDesc {
    const uint8_t* base;  // row-major bins of the storage block
    uint32_t stride;      // bytes per row (multiple of 16)
    uint32_t width;       // bytes per bin (1 or 2)
    uint32_t feat_begin;
    uint32_t n_feat;
    uint32_t local_bins;  // shared-memory bins of this tile
    uint32_t missing;     // missing-value sentinel of this width
    uint32_t chunk0;      // staged histogram: first 16-byte chunk of the record the tile reads
    uint32_t n_chunks;    // and the number of chunks (the features' bytes lie inside them)
};
struct TileFeat {
    uint32_t byte_off;    // byte offset of the feature inside a row record
    uint32_t local_off;   // first bin in the tile's shared histogram
    uint32_t nbins;
    uint32_t global_off;  // first bin in the node histogram
};

// Per-feature bin locator for partitions: the bin of row r is at
// base + r * stride + byte_off (row records, or a column-major copy with
// stride = width and byte_off = 0).
struct FeatLoc {
    const uint8_t* base;
    uint32_t stride;
    uint32_t byte_off;
    uint32_t width;
    uint32_t missing;
};

// Per-node split decision of the current level.
struct SplitDesc {
    int32_t child_slot;  // -1: terminal; else slot of the left child in the next level
    uint32_t feat;
    uint32_t bin;
    uint32_t flags;      // bit1 missing left, bit2 categorical
};

struct LevelArgs {
    // tree-wide
    uint32_t n_features;
    uint32_t max_leaves;
    uint32_t depth;
    uint32_t last_level;         // 1 when depth + 1 == max_depth (children are final leaves)
    ScoreParams sp;              // inv_g / inv_h are taken from `scales` on the device
    const double* scales;        // [2] quantizer scales of this round (device)
    const uint32_t* hoff;        // F+1 node-histogram offsets
    const uint8_t* enabled;      // per feature (colsample)
    const int8_t* mono;          // per feature monotone direction (may be null)
    const uint8_t* is_cat;       // per feature categorical flag (may be null)
    uint32_t max_onehot, max_cat_threshold;
    const FeatLoc* floc;
    const FeatLoc* floc_rec;     // the same features in the row records (k_tree_walk)
    uint32_t walk;               // depthwise: leaf values reach the margins by k_tree_walk, not per partition
    const uint8_t* walk_rec;     // k_tree_walk: the one record block holding every feature (stride <= 64), or null
    uint32_t walk_stride;
    // level buffers
    TreeState* st;
    NodeInfo* nodes;             // current level
    NodeInfo* next_nodes;        // next level
    const uint32_t* acc_list;    // current level: node index of each accumulate node
    const unsigned long long* acc_prefix;  // acc_count+1 row prefix
    uint32_t* next_acc_list;
    unsigned long long* next_acc_prefix;
    const uint32_t* chunk_prefix; // m+1 chunk prefix of the current level
    uint32_t* next_chunk_prefix;
    Pair* hist_acc;              // accumulate-node histograms (acc index slots)
    Pair* hist_cur;              // full histograms of this level (node slots)
    const Pair* hist_prev;       // full histograms of the previous level
    unsigned long long slot_pairs; // pairs per histogram slot (total bins; a rank's block when feature-sharded)
    uint32_t feat_lo, feat_hi;   // features this rank scores (all unless the split search is feature-sharded)
    uint32_t bin_lo;             // first bin of feat_lo in the node histograms (their slots hold bins from here)
    // the features of [feat_lo, feat_hi) split by search kernel: numeric ones of
    // up to 256 bins (a warp each, k_split_num) and the rest (a CTA each,
    // k_split_feat); null split_cta: every feature a CTA
    const uint32_t* split_num;
    uint32_t n_split_num;
    const uint32_t* split_cta;
    uint32_t n_split_cta;
    SplitRec* feat_best;         // [node * F + f]
    // category sets: cat_words 32-bit words each (>= 8; a bit per code, set =
    // right-going); codes at or beyond 32 * cat_words go left
    uint32_t cat_words;
    const uint32_t* cat_slot;    // per feature: its index among the categorical features
    uint32_t n_cat;              // categorical features
    uint32_t* feat_cats;         // [node * n_cat + cat_slot[f]][cat_words]
    SplitRec* node_best;         // [node]
    uint32_t* node_cats;         // [node][cat_words]
    SplitDesc* split;            // [node]
    uint32_t* chunk_left;        // per chunk left count
    uint32_t* chunk_off;         // per chunk left offset within its node
    uint8_t* dirflags;           // per 8 rows of a chunk: direction bits (null: recompute)
    uint32_t* node_left;         // per node left count (this rank)
    const uint32_t* node_left_global; // per node left count over all ranks
    const uint32_t* rows_cur;
    uint32_t* rows_next;
    float* pred;
    TreeRec* trec;
    uint32_t* tcats;             // [tree node][cat_words]
    const uint32_t* node_hist;   // lossguide: histogram-pool slot of each node (null: level slots)
    unsigned int* fuse;          // depthwise: zeroed counters; the one-CTA steps run in the last CTA
                                 // of the kernel before them (null: separate launches)
    unsigned long long* part_cnt; // depthwise: per node (left rows, right rows) reserved by k_part_level;
                                  // zero between levels
    unsigned long long* hist_zero; // depthwise: k_part_level zeroes the next level's accumulate
    unsigned long long hist_zero_words; // histograms (a multiple of 2 words), or nothing when null
};

#ifdef __CUDACC__
// Quantizer reciprocals of this round from the device scales (exact: the
// scales are powers of two).
__device__ __forceinline__ ScoreParams load_sp(const LevelArgs& a) {
    ScoreParams sp = a.sp;
    sp.inv_g = __ddiv_rn(1.0, a.scales[0]);
    sp.inv_h = __ddiv_rn(1.0, a.scales[1]);
    return sp;
}
#endif

struct GradArgs {
    uint32_t n;               // rows on this rank
    unsigned long long row0;  // global index of this rank's first row (sampling hash)
    unsigned long long sub_th, sub_seed, sub_tree;
    const float* label;
    const float* weight;      // may be null
    const float* pred;
    const float* host_exp;    // exact logistic: expf(-pred) computed by glibc on the host
    const float* gpair_in;    // exact reference path: f32 pairs from the host
    float* gpair_f32;         // scratch f32 pairs
    Pair* fixed;
    unsigned long long* sum;  // [2] root sum (mod 2^64)
    unsigned long long* maxbits; // [2] max |g|, |h| as double bit patterns
    const double* scales;     // [2]
    int objective;            // 0 squared error, 1 logistic
    const uint2* exptab;      // host-expf exception table (fexp.h), or null
    uint32_t exp_probes;      // longest probe sequence in exptab
};

// Host-side launchers (train_kernels.cu).
void launch_mask_max(const GradArgs& a, cudaStream_t s);
// mode 0: e from host_exp (or squared error), 1: fexp_core alone (fast mode),
// 2: the host C library's expf reproduced on the device (fexp_core + exptab).
void launch_gradient_max(const GradArgs& a, int mode, cudaStream_t s);
void launch_expf_emulate(const uint2* tab, uint32_t probes, uint32_t begin, uint32_t count, uint32_t* out,
                         cudaStream_t s);
void launch_gradient_quantize_exp(const GradArgs& a, cudaStream_t s);
void launch_quantize(const GradArgs& a, cudaStream_t s);
// objective.rs:1175-1219 softmax gradients of K classes: margins a.pred
// (K x a.n, class-major), labels, optional weights -> out (K x a.n f32 pairs,
// class-major).  fast: fexp_core alone; else the host expf (a.exptab).
void launch_softmax_gradients(const GradArgs& a, uint32_t K, float* out, int fast, cudaStream_t s);
void launch_device_scales(const unsigned long long* maxbits, unsigned long long n_rows, double* scales,
                          unsigned long long* err, cudaStream_t s);
// Exact mode: the reference's scales (qscale.h) and the error word (1: a
// non-finite bound, scales zero).
void launch_device_scales_exact(const unsigned long long* maxbits, unsigned long long n_rows,
                                const fbx::ScaleExc* exc, uint32_t n_exc, double* scales, unsigned long long* err,
                                cudaStream_t s);
void launch_quantizer_scales(const float* vals, uint64_t count, unsigned long long n_rows, const fbx::ScaleExc* exc,
                             uint32_t n_exc, double* out, cudaStream_t s);
void set_hist_smem_limit(int bytes);
void launch_hist(int width, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat, const uint32_t* rows,
                 const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                 const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                 unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s);
void set_hist_lpf_smem_limit(int bytes);
void launch_hist_lpf(int width, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat,
                     const uint32_t* rows, const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                     const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                     unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s);
// Lane-per-feature histogram with the rows' record chunks and gradient pairs
// staged in shared memory by a per-warp cp.async pipeline of `stages` (2 or
// 4) batches of kStageRows rows.  Shared memory: the tile's histogram planes
// plus hist_stage_bytes(n_chunks, stages).
constexpr uint32_t kStageRows = 8;
constexpr uint32_t kStageWarps = kHistLpfThreads / 32;
inline size_t hist_stage_bytes(uint32_t n_chunks, int stages) {
    return (size_t)kStageWarps * stages * kStageRows * (n_chunks * 16 + 16);
}
void set_hist_stage_smem_limit(int bytes);
// Wide features (441..1024 bins, 2-byte bins): the staged kernel with 8 lanes per
// row (4 rows per warp step), 8 features per tile.
constexpr uint32_t kWideLanes = 8;
inline size_t hist_wide_bytes(uint32_t max_bins) {  // four planes, bins + discard padded to 4
    return 4ull * (((max_bins + 1 + 3) / 4) * 4) * kWideLanes * 4;
}
void set_hist_wide_smem_limit(int bytes);
void launch_hist_wide(int stages, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat, const uint32_t* rows,
                      const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                      const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                      unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s);
void launch_hist_stage(int width, int stages, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat,
                       const uint32_t* rows, const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                       const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                       unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s);
void launch_split(const LevelArgs& a, uint32_t max_m, cudaStream_t s);
// k_split_feat, then per-node reduction and decisions in one launch (a.fuse set)
void launch_split_decide(const LevelArgs& a, uint32_t max_m, cudaStream_t s);
// Feature-sharded split search: merge the n_ranks gathered per-node winners
// (all_best / all_cats: [rank][max_m] records / sets) and decide the level.
void launch_merge_decide(const LevelArgs& a, const SplitRec* all_best, const uint32_t* all_cats, uint32_t n_ranks,
                         uint32_t max_m, cudaStream_t s);
void launch_part_count(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s);
void launch_part_scan(const LevelArgs& a, cudaStream_t s);
void launch_part_scatter(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s);
// Depthwise: one-pass partition of every node of the level, then the next
// level's tables (last CTA).  Needs a.fuse and a.part_cnt.
void launch_part_level(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s);
// Depthwise, last level: every row's final leaf value added to its margin
// (no partition into the children, no k_leaf_final after it).
void launch_part_final(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s);
void launch_leaf_final(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s);
// Every local row walks the finished tree (a.trec / a.tcats) on its record's
// bins and adds its leaf's value to its margin (training/mod.rs:5020-5063,
// one addition per row per tree as in the partition path).
// next_grad: also the next round's gradient pairs and their bounds from the
// new margins (gmode as launch_gradient_max's mode); null: the walk alone.
void launch_tree_walk(const LevelArgs& a, uint32_t n_rows, cudaStream_t s, const GradArgs* next_grad = nullptr,
                      int gmode = 0);
void launch_tree_init(const LevelArgs& a, uint32_t n_local, uint32_t n_global, const unsigned long long* root_sum,
                      cudaStream_t s);
void launch_iota(uint32_t* rows, uint32_t n, cudaStream_t s);
// p[0..n) = v
void launch_fill(float* p, uint64_t n, float v, cudaStream_t s);
void launch_records_to_columns(int width, const uint8_t* rec, uint32_t stride, uint64_t n_rows, uint32_t n_feats,
                               uint8_t* cols, cudaStream_t s);
void launch_transpose(int width, const uint8_t* src, uint8_t* dst, uint32_t n_rows, uint32_t n_feats,
                      uint32_t stride, uint64_t row0, cudaStream_t s);

}  // namespace fbg
