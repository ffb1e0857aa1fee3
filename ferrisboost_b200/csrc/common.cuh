// Shared device types and exact-arithmetic helpers for the FerrisBoost B200
// engine.  Every floating-point step that decides a split, a leaf value or a
// quantizer output uses explicit round-to-nearest intrinsics (no FMA
// contraction, no reassociation), so the device computes the same IEEE values
// as the reference CPU engine (src/training/split.rs, src/types.rs).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace fbg {

// Counts this library's kernel launches (fbgpu_launch_count).
void count_launch();

// Fixed-point gradient pair, modulo-2^64 arithmetic (types.rs:151-227).
struct Pair {
    long long g, h;
};
__device__ __host__ __forceinline__ Pair padd(Pair a, Pair b) {
    return {(long long)((unsigned long long)a.g + (unsigned long long)b.g),
            (long long)((unsigned long long)a.h + (unsigned long long)b.h)};
}
__device__ __host__ __forceinline__ Pair psub(Pair a, Pair b) {
    return {(long long)((unsigned long long)a.g - (unsigned long long)b.g),
            (long long)((unsigned long long)a.h - (unsigned long long)b.h)};
}
__device__ __host__ __forceinline__ bool peq(Pair a, Pair b) { return a.g == b.g && a.h == b.h; }

// Split-scoring parameters (TrainParams, types.rs:433-686).
struct ScoreParams {
    float lambda, gamma, mcw, alpha, mds, eta;
    double inv_g, inv_h;  // reciprocal quantizer scales (exact powers of two)
};

// Best candidate of one (node, feature) or one node.  flags: bit0 found,
// bit1 missing goes left, bit2 categorical.  `ord` orders equal gains the way
// the reference enumerates candidates (split.rs:254-270, 631-642).
struct SplitRec {
    float gain;
    uint32_t feat;
    uint32_t bin;
    uint32_t flags;
    Pair left, right;
    uint32_t ord;
    uint32_t pad[3];
};
static_assert(sizeof(SplitRec) == 64, "SplitRec layout");

// Per-node state of the level being grown (training/mod.rs:3239-3251 LevelNode).
struct NodeInfo {
    uint32_t start, len;   // span in the current row arena (this rank's rows)
    int32_t tree_id;       // index in the tree arrays
    int32_t parent_slot;   // -1: accumulate; else parent's slot in the previous level
    int32_t acc_slot;      // accumulate slot: own (accumulate) or the sibling's (subtract)
    float lower, upper;    // monotone bounds (split.rs:113-155)
    uint32_t len_global;   // rows of this node over all ranks
    Pair sum;              // node gradient sum including missing rows
};
static_assert(sizeof(NodeInfo) == 48, "NodeInfo layout");

// Device-resident tree record (model/tree.rs:52-79 Node).  flags: bit0 leaf,
// bit1 default_left, bit2 categorical.
struct TreeRec {
    int32_t left, right;
    uint32_t feat, bin;
    float gain, leaf, hess;
    uint32_t flags;
};
static_assert(sizeof(TreeRec) == 32, "TreeRec layout");

// Scalars shared by the level kernels of one tree (no host round trip).
struct TreeState {
    uint32_t m;            // nodes in the current level
    uint32_t n_tree_nodes; // nodes in the tree arrays
    uint32_t leaf_count;
    uint32_t acc_count;    // accumulate nodes in the current level
    unsigned long long acc_total;  // rows over the accumulate nodes
    uint32_t chunk_count;  // row chunks over the current level's nodes
    uint32_t kept;         // nodes split in the current level
    uint32_t error;        // nonzero: a kernel detected an inconsistency
    uint32_t pad0;
    // feature-sharded split search: pairs between two ranks' blocks of the
    // level's accumulate histograms (0 otherwise; see acc_bin)
    unsigned long long rank_stride;
    uint32_t pad[4];
};

__device__ __forceinline__ double to_f64(long long x, double inv) { return __dmul_rn(__ll2double_rn(x), inv); }

// split.rs:171-197 ThresholdL1 + CalcWeight, f64 then one rounding to f32.
__device__ __forceinline__ float xgb_weight(double g, double h, const ScoreParams& p) {
    if (h <= 0.0) return 0.0f;
    double a = (double)p.alpha;
    double t = g > a ? __dsub_rn(g, a) : (g < -a ? __dadd_rn(g, a) : 0.0);
    double dw = __ddiv_rn(-t, __dadd_rn(h, (double)p.lambda));
    if (p.mds != 0.0f && fabs(dw) > (double)p.mds) dw = copysign((double)p.mds, dw);
    return __double2float_rn(dw);
}
__device__ __forceinline__ float apply_bounds(float w, float lo, float hi) {
    return w < lo ? lo : (w > hi ? hi : w);
}
// split.rs:216-223 CalcGainGivenWeight (square in f32, the rest in f64).
__device__ __forceinline__ float gain_given_weight(double g, double h, float w, const ScoreParams& p) {
    if (h <= 0.0) return 0.0f;
    double sq = (double)__fmul_rn(w, w);
    double l1 = __dmul_rn(__dmul_rn(2.0, (double)p.alpha), (double)fabsf(w));
    double a = __dmul_rn(__dmul_rn(2.0, g), (double)w);
    double b = __dmul_rn(__dadd_rn(h, (double)p.lambda), sq);
    return __double2float_rn(-__dadd_rn(__dadd_rn(a, b), l1));
}
__device__ __forceinline__ float node_gain(Pair s, const ScoreParams& p, float lo, float hi) {
    double g = to_f64(s.g, p.inv_g), h = to_f64(s.h, p.inv_h);
    return gain_given_weight(g, h, apply_bounds(xgb_weight(g, h, p), lo, hi), p);
}
// split.rs:234-252 bounded_split_gain.  Returns false for an invalid candidate.
__device__ __forceinline__ bool split_gain(float parent, Pair l, Pair r, int constraint, float lo, float hi,
                                           const ScoreParams& p, float& out) {
    double lh = to_f64(l.h, p.inv_h), rh = to_f64(r.h, p.inv_h);
    double mcw = (double)p.mcw;
    if (!(lh > 0.0 && rh > 0.0 && lh >= mcw && rh >= mcw)) return false;
    double lg = to_f64(l.g, p.inv_g), rg = to_f64(r.g, p.inv_g);
    float wl = apply_bounds(xgb_weight(lg, lh, p), lo, hi);
    float wr = apply_bounds(xgb_weight(rg, rh, p), lo, hi);
    if ((constraint > 0 && wl > wr) || (constraint < 0 && wl < wr)) return false;
    float gain = __fadd_rn(gain_given_weight(lg, lh, wl, p), gain_given_weight(rg, rh, wr, p));
    float loss = __fsub_rn(gain, parent);
    out = __double2float_rn(__dsub_rn((double)loss, (double)p.gamma));
    return true;
}

// Candidate order: larger gain wins, equal gains go to the lower ordinal.
__device__ __forceinline__ bool rec_better(const SplitRec& a, const SplitRec& b) {
    if (!(a.flags & 1u)) return false;
    if (!(b.flags & 1u)) return true;
    return a.gain > b.gain || (a.gain == b.gain && a.ord < b.ord);
}

}  // namespace fbg

#define FB_CUDA_CHECK(expr)                                                        \
    do {                                                                           \
        cudaError_t _e = (expr);                                                   \
        if (_e != cudaSuccess) throw fbg::CudaError(_e, #expr, __FILE__, __LINE__); \
    } while (0)
