// Device sketch and quantization (sketch.cuh).
//
// The reference builds each feature's sketch sequentially
// (src/source/dense.rs:136-175, one thread per feature, no merging across
// row ranges): values are pushed in row order, every `limit` = max_bin x 16
// non-NaN values become a sorted, de-duplicated summary (build_summary,
// sketch.rs:305-329), and summaries enter a binary-counter hierarchy
// (insert_level, sketch.rs:161-180) where two summaries of the same level
// merge (merge_entries, :336-392) and are compressed back to `limit` entries
// (compress, :403-435).  collapse (:183-201) merges the occupied levels from
// the lowest up and compresses once; cuts (:236-275) pick equal-rank entries.
//
// That hierarchy is a fixed binary tree over the chunks: level l, node k
// covers chunks [k 2^l, (k+1) 2^l) and exists when (k+1) 2^l <= chunks.  The
// device builds it level by level, all nodes of a level (and all features)
// in parallel, and reproduces each sequential step exactly:
// - chunk summary: bitonic sort of the chunk's keys in shared memory, then
//   equal values grouped; with unit weights every rank is an exact integer.
// - merge: the output position and the rank shift of every entry follow
//   from two binary searches (a value is taken before the other list's
//   equal value when it comes from the first list), so each entry is
//   written independently with the same single f32 addition.
// - compress: target k picks taken_k = min(max(taken_{k-1} + 1, j_k),
//   ceil_k) with j_k the first index whose rmid reaches the target.  With
//   u_k = taken_k - k this is u_k = min(max(u_{k-1}, j_k - k), n - slots),
//   whose closed form is a prefix maximum, so all targets resolve in
//   parallel.  That form needs rmid non-decreasing, which the kernel checks;
//   if it does not hold, one thread runs the sequential loop instead.
// - cuts: the same binary search as the host's partition_point per target,
//   then the order-dependent de-duplication in one thread.
#include <omp.h>

#include <algorithm>
#include <mutex>
#include <cfloat>
#include <climits>
#include <cstring>
#include <numeric>
#include <stdexcept>

#include "ctx.h"
#include "sketch.cuh"

namespace fbg {
namespace {

constexpr int kSkThreads = 1024;
constexpr uint32_t kTileRows = 1024;   // rows per compaction tile
constexpr uint32_t kTileFeats = 8;     // features per compaction CTA (one warp each)

// Order-preserving map of non-NaN floats to u32 (-0 sorts just before +0);
// 0xffffffff (a NaN pattern) pads a partial chunk past every value.
__device__ __forceinline__ uint32_t f2key(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Exclusive sum over the CTA (blockDim a multiple of 32, <= 1024); sh holds
// 32 words.  Returns this thread's prefix; *total the CTA sum.  Ends synced.
__device__ uint32_t cta_excl_sum(uint32_t x, uint32_t* sh, uint32_t* total) {
    const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (uint32_t)o) v += y;
    }
    if (lane == 31u) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        uint32_t t = lane < nw ? sh[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= (uint32_t)o) t += y;
        }
        sh[lane] = t;
    }
    __syncthreads();
    const uint32_t before = w ? sh[w - 1] : 0u;
    *total = sh[nw - 1];
    __syncthreads();
    return before + v - x;
}

// Inclusive prefix maximum over the CTA; *total the CTA maximum.  Ends synced.
__device__ int cta_incl_max(int x, int* sh, int* total) {
    const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (uint32_t)o) v = max(v, y);
    }
    if (lane == 31u) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = lane < nw ? sh[lane] : INT_MIN;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= (uint32_t)o) t = max(t, y);
        }
        sh[lane] = t;
    }
    __syncthreads();
    const int r = w ? max(sh[w - 1], v) : v;
    *total = sh[nw - 1];
    __syncthreads();
    return r;
}

// First index with !(v[i] < x) over a non-decreasing array (the loop of
// libstdc++'s lower_bound / partition_point).
__device__ __forceinline__ uint32_t lower_bound_f(const float* v, uint32_t n, float x) {
    uint32_t first = 0, len = n;
    while (len > 0) {
        const uint32_t half = len >> 1;
        if (v[first + half] < x) { first += half + 1; len -= half + 1; } else { len = half; }
    }
    return first;
}
// First index with x < v[i].
__device__ __forceinline__ uint32_t upper_bound_f(const float* v, uint32_t n, float x) {
    uint32_t first = 0, len = n;
    while (len > 0) {
        const uint32_t half = len >> 1;
        if (!(x < v[first + half])) { first += half + 1; len -= half + 1; } else { len = half; }
    }
    return first;
}

// A summary in structure-of-arrays form: value, rmin, rmax (the weights of
// the reference's entries never decide anything and are not kept).
struct SumRef {
    const float* v;
    const float* lo;
    const float* hi;
};
struct SumMut {
    float* v;
    float* lo;
    float* hi;
    __device__ SumRef ref() const { return SumRef{v, lo, hi}; }
};
__device__ __forceinline__ SumMut sum_at(float* base_v, float* base_lo, float* base_hi, size_t off) {
    return SumMut{base_v + off, base_lo + off, base_hi + off};
}
// Entry::rmid (sketch.rs:43-45): 0.5 * (rmin + rmax) in f32.
__device__ __forceinline__ float rmid(const SumRef& s, uint32_t j) {
    return __fmul_rn(0.5f, __fadd_rn(s.lo[j], s.hi[j]));
}
__device__ __forceinline__ uint32_t lower_bound_rmid(const SumRef& s, uint32_t n, float t) {
    uint32_t first = 0, len = n;
    while (len > 0) {
        const uint32_t half = len >> 1;
        if (rmid(s, first + half) < t) { first += half + 1; len -= half + 1; } else { len = half; }
    }
    return first;
}

// merge_entries + dedup_same_value (sketch.rs:336-392).  Values inside A and
// inside B are strictly increasing, so only an A entry and an equal B entry
// can meet; the B entry folds into the A entry written just before it.
// tp: scratch of nb + 1 words.  Returns the merged size.
__device__ uint32_t cta_merge(SumRef A, uint32_t na, SumRef B, uint32_t nb, SumMut M, uint32_t* tp, uint32_t* sh) {
    uint32_t carry = 0;
    for (uint32_t base = 0; base < nb; base += blockDim.x) {
        const uint32_t j = base + threadIdx.x;
        uint32_t tied = 0;
        if (j < nb) {
            const float x = B.v[j];
            const uint32_t ub = upper_bound_f(A.v, na, x);
            tied = (ub > 0 && A.v[ub - 1] == x) ? 1u : 0u;
        }
        uint32_t tot;
        const uint32_t ex = cta_excl_sum(tied, sh, &tot);
        if (j < nb) tp[j] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) tp[nb] = carry;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < na; i += blockDim.x) {
        const float x = A.v[i], alo = A.lo[i], ahi = A.hi[i];
        const uint32_t lb = lower_bound_f(B.v, nb, x);  // B entries taken before A[i]
        const float pass_b = lb ? B.hi[lb - 1] : 0.0f;
        float lo = __fadd_rn(alo, pass_b), hi = __fadd_rn(ahi, pass_b);
        if (lb < nb && B.v[lb] == x) {  // B[lb] is taken right after A[i] with pass_a = A[i].rmax
            lo = fminf(lo, __fadd_rn(B.lo[lb], ahi));
            hi = fmaxf(hi, __fadd_rn(B.hi[lb], ahi));
        }
        const uint32_t o = i + lb - tp[lb];
        M.v[o] = x;
        M.lo[o] = lo;
        M.hi[o] = hi;
    }
    for (uint32_t j = threadIdx.x; j < nb; j += blockDim.x) {
        const float x = B.v[j];
        const uint32_t ub = upper_bound_f(A.v, na, x);  // A entries taken before B[j]
        if (ub > 0 && A.v[ub - 1] == x) continue;
        const float pass_a = ub ? A.hi[ub - 1] : 0.0f;
        const uint32_t o = j + ub - tp[j];
        M.v[o] = x;
        M.lo[o] = __fadd_rn(B.lo[j], pass_a);
        M.hi[o] = __fadd_rn(B.hi[j], pass_a);
    }
    const uint32_t m = na + nb - tp[nb];
    __syncthreads();
    return m;
}

// compress (sketch.rs:403-435) of M (m entries) into out, at most L entries.
// Returns the compressed size.  shi: 32 ints; sflag: one shared word.
__device__ uint32_t cta_prune(SumRef M, uint32_t m, SumMut out, uint32_t L, int* shi, uint32_t* sflag) {
    if (m <= L) {
        for (uint32_t j = threadIdx.x; j < m; j += blockDim.x) {
            out.v[j] = M.v[j];
            out.lo[j] = M.lo[j];
            out.hi[j] = M.hi[j];
        }
        __syncthreads();
        return m;
    }
    int bad = 0;
    for (uint32_t j = threadIdx.x; j + 1 < m; j += blockDim.x)
        if (rmid(M, j + 1) < rmid(M, j)) bad = 1;
    bad = __syncthreads_or(bad);
    const float total = M.hi[m - 1];
    const uint32_t slots = L - 1;
    if (!bad) {
        const int beta = (int)(m - slots);
        int carry = INT_MIN;
        for (uint32_t base = 1; base < slots; base += blockDim.x) {
            const uint32_t k = base + threadIdx.x;
            int a = INT_MIN;
            if (k < slots) {
                const float target = __fdiv_rn(__fmul_rn(total, (float)k), (float)slots);
                uint32_t j = lower_bound_rmid(M, m, target);
                if (j > m - 1) j = m - 1;
                a = (int)j - (int)k;
            }
            int tot;
            const int p = max(cta_incl_max(a, shi, &tot), carry);
            if (k < slots) {
                const int u = min(max(0, p), beta);
                const uint32_t t = k + (uint32_t)u;
                out.v[k] = M.v[t];
                out.lo[k] = M.lo[t];
                out.hi[k] = M.hi[t];
                if (k == slots - 1) *sflag = t;
            }
            carry = max(carry, tot);
        }
        if (threadIdx.x == 0) {
            out.v[0] = M.v[0];
            out.lo[0] = M.lo[0];
            out.hi[0] = M.hi[0];
        }
        __syncthreads();
        const uint32_t last = *sflag;
        uint32_t n_out = slots;
        if (last < m - 1) {
            if (threadIdx.x == 0) {
                out.v[slots] = M.v[m - 1];
                out.lo[slots] = M.lo[m - 1];
                out.hi[slots] = M.hi[m - 1];
            }
            n_out = slots + 1;
        }
        __syncthreads();
        return n_out;
    }
    // rmid not monotone: the reference's loop, one thread
    if (threadIdx.x == 0) {
        uint32_t c = 0, taken = 0;
        out.v[c] = M.v[0]; out.lo[c] = M.lo[0]; out.hi[c] = M.hi[0]; c++;
        for (uint32_t k = 1; k < slots; k++) {
            const float target = __fdiv_rn(__fmul_rn(total, (float)k), (float)slots);
            uint32_t j = taken + 1;
            while (j < m - 1 && rmid(M, j) < target) j++;
            const uint32_t ceiling = m - 1 - (slots - 1 - k);
            j = min(max(j, taken + 1), ceiling);
            if (j > taken) {
                out.v[c] = M.v[j]; out.lo[c] = M.lo[j]; out.hi[c] = M.hi[j]; c++;
                taken = j;
            }
        }
        if (taken < m - 1) { out.v[c] = M.v[m - 1]; out.lo[c] = M.lo[m - 1]; out.hi[c] = M.hi[m - 1]; c++; }
        *sflag = c;
    }
    __syncthreads();
    const uint32_t n_out = *sflag;
    __syncthreads();
    return n_out;
}

// sketch.rs:281-302 midpoint.
__device__ __forceinline__ float midpoint(float a, float b) {
    const float d = __fsub_rn(b, a);
    const float m = isfinite(d) ? __fadd_rn(a, __fmul_rn(d, 0.5f)) : __fadd_rn(__fmul_rn(a, 0.5f), __fmul_rn(b, 0.5f));
    return m <= a ? b : m;
}

// --------------------------------------------------------------- kernels
// Non-NaN values per (feature, row tile).  Warp j of the CTA counts feature
// g0 + j of the batch over the tile's rows.
__global__ void __launch_bounds__(256) k_valid_count(const float* __restrict__ X, uint64_t n, uint64_t rs, uint64_t cs,
                                                     const uint32_t* __restrict__ feats, uint32_t nbf,
                                                     uint32_t n_tiles, uint32_t* __restrict__ cnt) {
    const uint32_t tile = blockIdx.x, lane = threadIdx.x & 31u, j = blockIdx.y * kTileFeats + (threadIdx.x >> 5);
    if (j >= nbf) return;
    const uint64_t r0 = (uint64_t)tile * kTileRows;
    const uint32_t rows = (uint32_t)min((uint64_t)kTileRows, n - r0);
    const uint32_t f = feats[j];
    uint32_t c = 0;
    for (uint32_t r = lane; r < rows; r += 32) c += isnan(X[(r0 + r) * rs + f * cs]) ? 0u : 1u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) cnt[(size_t)j * n_tiles + tile] = c;
}

// Stable compaction: the non-NaN values of batch feature j, in row order, to
// vals[vbase[j] + ...]; tile_off[j * n_tiles + t] = values before tile t.
__global__ void __launch_bounds__(256) k_compact(const float* __restrict__ X, uint64_t n, uint64_t rs, uint64_t cs,
                                                 const uint32_t* __restrict__ feats, uint32_t nbf, uint32_t n_tiles,
                                                 const unsigned long long* __restrict__ vbase,
                                                 const uint32_t* __restrict__ tile_off, float* __restrict__ vals) {
    const uint32_t tile = blockIdx.x, lane = threadIdx.x & 31u, j = blockIdx.y * kTileFeats + (threadIdx.x >> 5);
    if (j >= nbf) return;
    const uint64_t r0 = (uint64_t)tile * kTileRows;
    const uint32_t rows = (uint32_t)min((uint64_t)kTileRows, n - r0);
    const uint32_t f = feats[j];
    float* out = vals + vbase[j] + tile_off[(size_t)j * n_tiles + tile];
    uint32_t pos = 0;
    for (uint32_t r = 0; r < rows; r += 32) {
        const uint32_t rr = r + lane;
        const float x = rr < rows ? X[(r0 + rr) * rs + f * cs] : __int_as_float(0x7fc00000);
        const bool ok = !isnan(x);
        const uint32_t bal = __ballot_sync(0xffffffffu, ok);
        if (ok) out[pos + __popc(bal & ((1u << lane) - 1u))] = x;
        pos += __popc(bal);
    }
}

struct SlotArrays {
    float* v;
    float* lo;
    float* hi;
    uint32_t* count;
    uint32_t L;
};

// The bitonic network of k_chunk_summary over 4096 keys with 1024 threads,
// thread t holding keys 4t .. 4t + 3 in registers: a compare-exchange at
// distance j < 4 stays in the thread, 4 <= j <= 64 pairs lanes of one warp
// (shuffles), and only j >= 128 goes through shared memory (15 of the 78
// stages).  Every stage compares the same pairs in the same direction as the
// shared-memory loop, so the sorted keys are the same.  Ends with the keys
// in keys[0 .. 4096) and the CTA synced.
__device__ void bitonic_sort_4096(const float* __restrict__ src, uint32_t cnt, uint32_t* keys) {
    const uint32_t t = threadIdx.x, lane = t & 31u;
    uint32_t x[4];
#pragma unroll
    for (uint32_t e = 0; e < 4; e++) {
        const uint32_t i = 4 * t + e;
        x[e] = i < cnt ? f2key(src[i]) : 0xffffffffu;
    }
    for (uint32_t k = 2; k <= 4096; k <<= 1) {
        uint32_t j = k >> 1;
        if (j >= 128) {
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) keys[4 * t + e] = x[e];
            __syncthreads();
            for (; j >= 128; j >>= 1) {
#pragma unroll
                for (uint32_t h = 0; h < 2; h++) {
                    const uint32_t p = t + h * 1024u;
                    const uint32_t i = 2 * p - (p & (j - 1)), ixj = i + j;
                    const uint32_t a = keys[i], b = keys[ixj];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) { keys[i] = b; keys[ixj] = a; }
                }
                __syncthreads();
            }
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) x[e] = keys[4 * t + e];
        }
        for (; j >= 4; j >>= 1) {
            const uint32_t d = j >> 2;  // partner lane offset
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) {
                const uint32_t i = 4 * t + e;
                const uint32_t y = __shfl_xor_sync(0xffffffffu, x[e], d);
                const bool lower = (i & j) == 0, up = (i & k) == 0;
                x[e] = (lower == up) ? min(x[e], y) : max(x[e], y);
            }
        }
        (void)lane;
        for (; j >= 1; j >>= 1) {
#pragma unroll
            for (uint32_t e = 0; e < 4; e++) {
                if (e & j) continue;
                const uint32_t i = 4 * t + e;
                const bool up = (i & k) == 0;
                const uint32_t a = x[e], b = x[e + j];
                if ((a > b) == up) { x[e] = b; x[e + j] = a; }
            }
        }
    }
#pragma unroll
    for (uint32_t e = 0; e < 4; e++) keys[4 * t + e] = x[e];
    __syncthreads();
}

// build_summary (sketch.rs:305-329) of one chunk with unit weights: sorted,
// equal values grouped, rmin = values before the group, rmax = rmin + count.
__global__ void __launch_bounds__(kSkThreads) k_chunk_summary(const float* __restrict__ vals,
                                                              const unsigned long long* __restrict__ vbase,
                                                              const unsigned long long* __restrict__ nval,
                                                              const uint32_t* __restrict__ task_feat,
                                                              const uint32_t* __restrict__ task_chunk,
                                                              const uint32_t* __restrict__ sbase, SlotArrays S) {
    extern __shared__ uint32_t keys[];
    __shared__ uint32_t sh[32];
    const uint32_t L = S.L;
    const uint32_t jb = task_feat[blockIdx.x], c = task_chunk[blockIdx.x];
    const unsigned long long first = (unsigned long long)c * L;
    const uint32_t cnt = (uint32_t)min((unsigned long long)L, nval[jb] - first);
    uint32_t P = 1;
    while (P < cnt) P <<= 1;
    const float* src = vals + vbase[jb] + first;
    if (P == 4 * kSkThreads && blockDim.x == kSkThreads) {
        bitonic_sort_4096(src, cnt, keys);
    } else {
    for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) keys[i] = i < cnt ? f2key(src[i]) : 0xffffffffu;
    __syncthreads();
    for (uint32_t k = 2; k <= P; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t p = threadIdx.x; p < (P >> 1); p += blockDim.x) {
                // p = q j + r (r < j, j a power of two): i = 2 q j + r = 2 p - r
                const uint32_t i = 2 * p - (p & (j - 1)), ixj = i + j;
                const uint32_t a = keys[i], b = keys[ixj];
                const bool up = (i & k) == 0;
                if ((a > b) == up) { keys[i] = b; keys[ixj] = a; }
            }
            __syncthreads();
        }
    }
    }
    const uint32_t slot = sbase[jb] + c;
    float* ov = S.v + (size_t)slot * L;
    float* olo = S.lo + (size_t)slot * L;
    float* ohi = S.hi + (size_t)slot * L;
    const uint32_t ipt = (cnt + blockDim.x - 1) / blockDim.x;
    const uint32_t b0 = min(threadIdx.x * ipt, cnt), b1 = min(b0 + ipt, cnt);
    uint32_t starts = 0;
    for (uint32_t i = b0; i < b1; i++) starts += (i == 0 || key2f(keys[i]) != key2f(keys[i - 1])) ? 1u : 0u;
    uint32_t total;
    uint32_t g = cta_excl_sum(starts, sh, &total);
    for (uint32_t i = b0; i < b1; i++) {
        const float x = key2f(keys[i]);
        if (i == 0 || x != key2f(keys[i - 1])) {
            ov[g] = x;
            olo[g] = (float)i;
            g++;
        }
        if (i + 1 == cnt || key2f(keys[i + 1]) != x) ohi[g - 1] = (float)(i + 1);
    }
    if (threadIdx.x == 0) S.count[slot] = total;
}

// One level of the hierarchy: slot left <- compress(merge(left, right)).
// Persistent CTAs; each owns 3 x 2L floats + (L + 1) words of scratch.
__global__ void __launch_bounds__(kSkThreads) k_merge_level(SlotArrays S, const uint32_t* __restrict__ task_left,
                                                            const uint32_t* __restrict__ task_right, uint32_t n_tasks,
                                                            float* scratch, uint32_t* tscratch) {
    __shared__ uint32_t sh[32];
    __shared__ int shi[32];
    __shared__ uint32_t sflag;
    const uint32_t L = S.L;
    const size_t cap = 2 * (size_t)L;
    SumMut M = sum_at(scratch, scratch + cap, scratch + 2 * cap, (size_t)blockIdx.x * 3 * cap);
    uint32_t* tp = tscratch + (size_t)blockIdx.x * (L + 1);
    for (uint32_t t = blockIdx.x; t < n_tasks; t += gridDim.x) {
        const uint32_t a = task_left[t], b = task_right[t];
        const uint32_t na = S.count[a], nb = S.count[b];
        SumMut A = sum_at(S.v, S.lo, S.hi, (size_t)a * L);
        SumMut B = sum_at(S.v, S.lo, S.hi, (size_t)b * L);
        const uint32_t m = cta_merge(A.ref(), na, B.ref(), nb, M, tp, sh);
        const uint32_t no = cta_prune(M.ref(), m, A, L, shi, &sflag);
        if (threadIdx.x == 0) S.count[a] = no;
        __syncthreads();
    }
}

// The same level with each task's two summaries and its merge held in shared
// memory (13 L + 1 words: L <= kMergeSmemMaxL), so the binary searches of the
// merge and the compress read shared memory instead of L2.  One CTA per SM.
constexpr uint32_t kMergeSmemMaxL = 4096;
__global__ void __launch_bounds__(kSkThreads) k_merge_level_smem(SlotArrays S, const uint32_t* __restrict__ task_left,
                                                                 const uint32_t* __restrict__ task_right,
                                                                 uint32_t n_tasks) {
    extern __shared__ float msm[];
    __shared__ uint32_t sh[32];
    __shared__ int shi[32];
    __shared__ uint32_t sflag;
    const uint32_t L = S.L;
    SumMut As = sum_at(msm, msm + L, msm + 2 * L, 0);
    SumMut Bs = sum_at(msm + 3 * L, msm + 4 * L, msm + 5 * L, 0);
    SumMut M = sum_at(msm + 6 * L, msm + 8 * L, msm + 10 * L, 0);
    uint32_t* tp = reinterpret_cast<uint32_t*>(msm + 12 * L);
    for (uint32_t t = blockIdx.x; t < n_tasks; t += gridDim.x) {
        const uint32_t a = task_left[t], b = task_right[t];
        const uint32_t na = S.count[a], nb = S.count[b];
        SumMut A = sum_at(S.v, S.lo, S.hi, (size_t)a * L);
        const SumRef B = sum_at(S.v, S.lo, S.hi, (size_t)b * L).ref();
        for (uint32_t i = threadIdx.x; i < na; i += blockDim.x) {
            As.v[i] = A.v[i]; As.lo[i] = A.lo[i]; As.hi[i] = A.hi[i];
        }
        for (uint32_t i = threadIdx.x; i < nb; i += blockDim.x) {
            Bs.v[i] = B.v[i]; Bs.lo[i] = B.lo[i]; Bs.hi[i] = B.hi[i];
        }
        __syncthreads();
        const uint32_t m = cta_merge(As.ref(), na, Bs.ref(), nb, M, tp, sh);
        const uint32_t no = cta_prune(M.ref(), m, A, L, shi, &sflag);
        if (threadIdx.x == 0) S.count[a] = no;
        __syncthreads();
    }
}

// collapse (sketch.rs:183-201) of one feature, then cuts (:236-275).
// list[list_off[j] ..] are the slots of the occupied levels, lowest first;
// each feature owns two merge buffers and a tied-prefix buffer of cap[j].
__global__ void __launch_bounds__(kSkThreads) k_collapse_cuts(SlotArrays S, const uint32_t* __restrict__ list_off,
                                                              const uint32_t* __restrict__ list,
                                                              const unsigned long long* __restrict__ buf_off,
                                                              const uint32_t* __restrict__ buf_cap, float* buf,
                                                              uint32_t* tbuf, float* fin, uint32_t max_bin,
                                                              float* cuts_out, uint32_t* ncuts_out) {
    __shared__ uint32_t sh[32];
    __shared__ int shi[32];
    __shared__ uint32_t sflag;
    __shared__ float cand[1024];
    const uint32_t j = blockIdx.x, L = S.L;
    const uint32_t k0 = list_off[j], k1 = list_off[j + 1];
    if (k0 == k1) {
        if (threadIdx.x == 0) ncuts_out[j] = 0;
        return;
    }
    const size_t cap = buf_cap[j];
    float* base = buf + buf_off[j];
    SumMut bufs[2] = {sum_at(base, base + cap, base + 2 * cap, 0), sum_at(base, base + cap, base + 2 * cap, 3 * cap)};
    uint32_t* tp = tbuf + buf_off[j] / 6 + j;  // cap + 1 words per feature
    SumRef acc = sum_at(S.v, S.lo, S.hi, (size_t)list[k0] * L).ref();
    uint32_t na = S.count[list[k0]];
    for (uint32_t k = k0 + 1; k < k1; k++) {
        const uint32_t s = list[k];
        SumMut dst = bufs[(k - k0 - 1) & 1];
        na = cta_merge(acc, na, sum_at(S.v, S.lo, S.hi, (size_t)s * L).ref(), S.count[s], dst, tp, sh);
        acc = dst.ref();
    }
    SumMut E = sum_at(fin, fin + (size_t)gridDim.x * L, fin + 2 * (size_t)gridDim.x * L, (size_t)j * L);
    const uint32_t e = cta_prune(acc, na, E, L, shi, &sflag);
    const SumRef R = E.ref();
    const uint32_t n_cuts = max_bin >= 1 ? max_bin - 1 : 0;
    float* out = cuts_out + (size_t)j * (max_bin ? max_bin : 1);
    if (n_cuts == 0 || e == 0) {
        if (threadIdx.x == 0) ncuts_out[j] = 0;
        return;
    }
    if (e <= n_cuts) {
        for (uint32_t i = threadIdx.x; i + 1 < e; i += blockDim.x) out[i] = midpoint(R.v[i], R.v[i + 1]);
        if (threadIdx.x == 0) ncuts_out[j] = e - 1;
        return;
    }
    const float total = R.hi[e - 1];
    for (uint32_t k = 1 + threadIdx.x; k <= n_cuts; k += blockDim.x) {
        const float target = __fdiv_rn(__fmul_rn(total, (float)k), (float)max_bin);
        uint32_t idx = lower_bound_rmid(R, e, target);
        if (idx > e - 1) idx = e - 1;
        cand[k - 1] = R.v[idx];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t c = 0;
        for (uint32_t k = 0; k < n_cuts; k++) {
            const float v = cand[k];
            if (c == 0 || v > out[c - 1]) out[c++] = v;
        }
        ncuts_out[j] = c;
    }
}

// categorical.rs:264-266 scan: largest valid code of batch feature
// blockIdx.y; invalid codes (negative, > 65533 or fractional) flag the
// feature.
__global__ void __launch_bounds__(256) k_cat_scan(const float* __restrict__ X, uint64_t n, uint64_t rs, uint64_t cs,
                                                  const uint32_t* __restrict__ feats, int* max_code,
                                                  unsigned int* bad) {
    __shared__ int smax[8];
    __shared__ int sbad[8];
    const uint32_t j = blockIdx.y, f = feats[j];
    int mx = -1, b = 0;
    for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < n; r += (uint64_t)gridDim.x * blockDim.x) {
        const float x = X[r * rs + f * cs];
        if (isnan(x)) continue;
        if (x < 0.0f || x > 65533.0f || x != truncf(x)) b = 1;
        else mx = max(mx, (int)x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        b |= __shfl_xor_sync(0xffffffffu, b, o);
    }
    if ((threadIdx.x & 31u) == 0) { smax[threadIdx.x >> 5] = mx; sbad[threadIdx.x >> 5] = b; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) { mx = max(mx, smax[w]); b |= sbad[w]; }
        if (mx >= 0) atomicMax(&max_code[j], mx);
        if (b) atomicOr(&bad[j], 1u);
    }
}

// Which features hold a NaN: one coalesced pass over the matrix; a NaN sets
// its feature's flag with a plain store (every writer stores 1).
__global__ void __launch_bounds__(256) k_nan_scan(const float* __restrict__ X, uint64_t n, uint32_t F, uint64_t cs,
                                                  uint8_t* __restrict__ flags) {
    const uint64_t total = n * F;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x)
        if (isnan(X[e])) flags[cs == 1 ? (uint32_t)(e % F) : (uint32_t)(e / n)] = 1;
}

// dense.rs:288-308 quantize_dense into row records, one warp per row: lane i
// bins block feature i (+32, +64, +96), so writes of the record are
// contiguous, and so are reads of a row-major X (a column-major X is read a
// 32-byte sector per column, shared by the 8 consecutive rows of a CTA).
template <int W>
__global__ void __launch_bounds__(256) k_bin_block(const float* __restrict__ X, uint64_t n, uint64_t rs, uint64_t cs,
                                                   const uint32_t* __restrict__ bfeats, uint32_t nf,
                                                   const float* __restrict__ cuts, const uint32_t* __restrict__ off,
                                                   const uint8_t* __restrict__ cat, uint8_t* __restrict__ dst,
                                                   uint32_t stride, unsigned int* reserved) {
    constexpr uint32_t miss = W == 2 ? 65535u : 255u;
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t fid[4], o[4], nc[4];
    bool iscat[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const uint32_t i = lane + 32u * q;
        fid[q] = i < nf ? bfeats[i] : 0u;
        o[q] = i < nf ? off[fid[q]] : 0u;
        nc[q] = i < nf ? off[fid[q] + 1] - o[q] : 0u;
        iscat[q] = i < nf ? cat[fid[q]] != 0 : false;
    }
    int res = 0;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t r = blockIdx.x * (uint64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
        uint8_t* rec = dst + r * stride;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint32_t i = lane + 32u * q;
            if (i >= nf) break;
            const float x = X[r * rs + fid[q] * cs];
            if (x == FLT_MAX || isinf(x)) res = 1;
            uint32_t bin;
            if (isnan(x)) bin = miss;
            else if (iscat[q]) bin = (x >= 0.0f && x < (float)(nc[q] + 1)) ? (uint32_t)x : miss - 1;
            else bin = upper_bound_f(cuts + o[q], nc[q], x);
            if (W == 2) reinterpret_cast<uint16_t*>(rec)[i] = (uint16_t)bin;
            else rec[i] = (uint8_t)bin;
        }
    }
    if (__syncthreads_or(res) && threadIdx.x == 0) atomicOr(reserved, 1u);
}

template <class T> void upload(DevMem& d, const std::vector<T>& h, cudaStream_t s) {
    d.alloc(std::max<size_t>(h.size(), 1) * sizeof(T));
    if (!h.empty()) FB_CUDA_CHECK(cudaMemcpyAsync(d.p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice, s));
}

}  // namespace

DeviceMatrix::DeviceMatrix(const HostMatrix& X_host, uint64_t n, uint32_t F, cudaStream_t stream, int threads)
    : n_(n), F_(F), rs_(X_host.rs), cs_(X_host.cs), s_(stream) {
    const int nth = threads > 0 ? threads : omp_get_max_threads();
    if (!((rs_ == F && cs_ == 1) || (rs_ == 1 && cs_ == n)))
        throw std::invalid_argument("DeviceMatrix: the host matrix must be contiguous row-major or column-major");
    const size_t bytes = (size_t)n * F * sizeof(float);
    x_ = static_cast<float*>(dev_alloc(std::max<size_t>(bytes, 16), &x_cap_));
    // pageable source: pinned staging in slabs, two buffers so the host copy
    // of one slab overlaps the transfer of the other.  The two 64 MiB buffers
    // are allocated once per process and kept (pinned allocation costs tens
    // of milliseconds); one upload uses them at a time.
    const size_t slab = std::min<size_t>(bytes, 64ull << 20);
    if (bytes) {
        static std::mutex stage_mu;
        static PinnedMem stage[2];
        std::lock_guard<std::mutex> stage_lock(stage_mu);
        cudaEvent_t done[2];
        for (int i = 0; i < 2; i++) {
            stage[i].reserve(64ull << 20);
            FB_CUDA_CHECK(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        const char* src = reinterpret_cast<const char*>(X_host.p);
        int k = 0;
        bool used[2] = {false, false};
        try {
            for (size_t off = 0; off < bytes; off += slab, k ^= 1) {
                const size_t len = std::min(slab, bytes - off);
                if (used[k]) FB_CUDA_CHECK(cudaEventSynchronize(done[k]));
                char* dst = stage[k].as<char>();
#pragma omp parallel for schedule(static) num_threads(nth)
                for (int64_t p = 0; p < (int64_t)len; p += (1 << 20))
                    std::memcpy(dst + p, src + off + p, std::min<size_t>(1 << 20, len - (size_t)p));
                FB_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<char*>(x_) + off, dst, len, cudaMemcpyHostToDevice, s_));
                FB_CUDA_CHECK(cudaEventRecord(done[k], s_));
                used[k] = true;
            }
            FB_CUDA_CHECK(cudaStreamSynchronize(s_));
        } catch (...) {
            cudaStreamSynchronize(s_);
            for (auto& e : done) cudaEventDestroy(e);
            dev_free(x_, x_cap_);
            x_ = nullptr;
            throw;
        }
        for (auto& e : done) cudaEventDestroy(e);
    }
}

std::vector<uint8_t> DeviceMatrix::nan_features() {
    DevMem d_flags;
    d_flags.alloc(std::max<uint32_t>(F_, 1));
    FB_CUDA_CHECK(cudaMemsetAsync(d_flags.p, 0, std::max<uint32_t>(F_, 1), s_));
    if (n_ && F_) {
        const uint64_t blocks = std::min<uint64_t>(ceil_div((uint64_t)n_ * F_, 256), 148ull * 16);
        count_launch();
        k_nan_scan<<<(unsigned)blocks, 256, 0, s_>>>(x_, n_, F_, cs_, d_flags.as<uint8_t>());
        FB_CUDA_CHECK(cudaGetLastError());
    }
    std::vector<uint8_t> out(F_);
    if (F_) FB_CUDA_CHECK(cudaMemcpyAsync(out.data(), d_flags.p, F_, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    return out;
}

DeviceMatrix::~DeviceMatrix() {
    if (x_) {
        cudaStreamSynchronize(s_);
        dev_free(x_, x_cap_);
    }
}

void DeviceMatrix::numeric_cuts(uint32_t max_bin, const std::vector<uint32_t>& feats,
                                std::vector<std::vector<float>>& per) {
    per.assign(feats.size(), {});
    if (feats.empty() || n_ == 0 || max_bin <= 1) return;  // no cuts (sketch.rs:245-248)
    const uint32_t L = std::max<uint32_t>(max_bin * 16u, 32u);  // sketch.rs:73 SKETCH_RATIO
    if (L > kSketchMaxLimit) throw InputError("the device sketch supports max_bin up to 1024");
    uint32_t P = 1;
    while (P < L) P <<= 1;
    // the attribute is per device; setting it again is harmless
    FB_CUDA_CHECK(cudaFuncSetAttribute(k_chunk_summary, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(kSketchMaxLimit * sizeof(uint32_t))));
    const uint32_t n_tiles = ceil_div(n_, kTileRows);
    // features per batch: values (4 B) + chunk slots (12 B) per row, bounded
    // by a quarter of the free device memory
    size_t free_b = 0, total_b = 0;
    FB_CUDA_CHECK(cudaMemGetInfo(&free_b, &total_b));
    const size_t per_feat = (size_t)n_ * 16 + (size_t)L * 48 + (size_t)n_tiles * 8 + 4096;
    const size_t budget = std::min<size_t>(free_b / 4, 16ull << 30);
    const size_t bsz = std::max<size_t>(1, std::min<size_t>(feats.size(), budget / per_feat));

    for (size_t b0 = 0; b0 < feats.size(); b0 += bsz) {
        const uint32_t nbf = (uint32_t)std::min(bsz, feats.size() - b0);
        std::vector<uint32_t> bf(feats.begin() + b0, feats.begin() + b0 + nbf);
        DevMem d_feats, d_cnt;
        upload(d_feats, bf, s_);
        d_cnt.alloc((size_t)nbf * n_tiles * 4);
        dim3 tg(n_tiles, ceil_div(nbf, kTileFeats));
        count_launch();
        k_valid_count<<<tg, 256, 0, s_>>>(x_, n_, rs_, cs_, d_feats.as<uint32_t>(), nbf, n_tiles, d_cnt.as<uint32_t>());
        FB_CUDA_CHECK(cudaGetLastError());
        std::vector<uint32_t> cnt((size_t)nbf * n_tiles);
        FB_CUDA_CHECK(cudaMemcpyAsync(cnt.data(), d_cnt.p, cnt.size() * 4, cudaMemcpyDeviceToHost, s_));
        FB_CUDA_CHECK(cudaStreamSynchronize(s_));
        std::vector<unsigned long long> vbase(nbf + 1, 0), nval(nbf, 0);
        std::vector<uint32_t> tile_off(cnt.size()), sbase(nbf + 1, 0), nch(nbf, 0);
        for (uint32_t j = 0; j < nbf; j++) {
            uint32_t acc = 0;
            for (uint32_t t = 0; t < n_tiles; t++) {
                tile_off[(size_t)j * n_tiles + t] = acc;
                acc += cnt[(size_t)j * n_tiles + t];
            }
            nval[j] = acc;
            vbase[j + 1] = vbase[j] + acc;
            nch[j] = ceil_div(acc, L);
            sbase[j + 1] = sbase[j] + nch[j];
        }
        const uint32_t n_slots = sbase[nbf];
        DevMem d_vbase, d_nval, d_toff, d_vals, d_sbase;
        upload(d_vbase, vbase, s_);
        upload(d_nval, nval, s_);
        upload(d_toff, tile_off, s_);
        upload(d_sbase, sbase, s_);
        d_vals.alloc(std::max<size_t>(vbase[nbf], 1) * 4);
        count_launch();
        k_compact<<<tg, 256, 0, s_>>>(x_, n_, rs_, cs_, d_feats.as<uint32_t>(), nbf, n_tiles,
                                      d_vbase.as<unsigned long long>(), d_toff.as<uint32_t>(), d_vals.as<float>());
        FB_CUDA_CHECK(cudaGetLastError());
        if (n_slots == 0) {  // every batch feature is all-NaN: no cuts
            FB_CUDA_CHECK(cudaStreamSynchronize(s_));
            continue;
        }

        // level 0: one summary per chunk
        std::vector<uint32_t> tf(n_slots), tc(n_slots);
        for (uint32_t j = 0; j < nbf; j++)
            for (uint32_t c = 0; c < nch[j]; c++) { tf[sbase[j] + c] = j; tc[sbase[j] + c] = c; }
        DevMem d_tf, d_tc, d_sv, d_scount;
        upload(d_tf, tf, s_);
        upload(d_tc, tc, s_);
        d_sv.alloc((size_t)n_slots * L * 12);
        d_scount.alloc((size_t)n_slots * 4);
        SlotArrays S{d_sv.as<float>(), d_sv.as<float>() + (size_t)n_slots * L,
                     d_sv.as<float>() + 2 * (size_t)n_slots * L, d_scount.as<uint32_t>(), L};
        count_launch();
        k_chunk_summary<<<n_slots, kSkThreads, P * sizeof(uint32_t), s_>>>(
            d_vals.as<float>(), d_vbase.as<unsigned long long>(), d_nval.as<unsigned long long>(),
            d_tf.as<uint32_t>(), d_tc.as<uint32_t>(), d_sbase.as<uint32_t>(), S);
        FB_CUDA_CHECK(cudaGetLastError());
        FB_CUDA_CHECK(cudaStreamSynchronize(s_));
        d_vals.release();

        // levels 1..: node k of level l lives in the slot of its first chunk
        const uint32_t max_ch = *std::max_element(nch.begin(), nch.end());
        const uint32_t grid_cap = 148u * 2u;
        // shared-memory merges when the summaries fit (max_bin <= 256)
        int dev = 0, sms = 148, optin = 0;
        FB_CUDA_CHECK(cudaGetDevice(&dev));
        FB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        FB_CUDA_CHECK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        size_t merge_smem = (size_t)(13 * L + 1) * 4;
        if (L > kMergeSmemMaxL || merge_smem + 1024 > (size_t)optin) merge_smem = 0;
        if (merge_smem)
            FB_CUDA_CHECK(cudaFuncSetAttribute(k_merge_level_smem, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)merge_smem));
        DevMem d_scr, d_tscr, d_tl, d_tr;
        for (uint32_t l = 1; (1ull << l) <= max_ch; l++) {
            std::vector<uint32_t> tl, tr;
            for (uint32_t j = 0; j < nbf; j++)
                for (uint32_t k = 0; k < (nch[j] >> l); k++) {
                    tl.push_back(sbase[j] + (k << l));
                    tr.push_back(sbase[j] + (k << l) + (1u << (l - 1)));
                }
            const uint32_t nt = (uint32_t)tl.size();
            const uint32_t grid = std::min(nt, grid_cap);
            if (!merge_smem && d_scr.bytes < (size_t)grid * 6 * L * 4) d_scr.alloc((size_t)grid * 6 * L * 4);
            if (!merge_smem && d_tscr.bytes < (size_t)grid * (L + 1) * 4) d_tscr.alloc((size_t)grid * (L + 1) * 4);
            upload(d_tl, tl, s_);
            upload(d_tr, tr, s_);
            count_launch();
            if (merge_smem)
                k_merge_level_smem<<<std::min(nt, (uint32_t)sms), kSkThreads, merge_smem, s_>>>(
                    S, d_tl.as<uint32_t>(), d_tr.as<uint32_t>(), nt);
            else
                k_merge_level<<<grid, kSkThreads, 0, s_>>>(S, d_tl.as<uint32_t>(), d_tr.as<uint32_t>(), nt,
                                                           d_scr.as<float>(), d_tscr.as<uint32_t>());
            FB_CUDA_CHECK(cudaGetLastError());
            FB_CUDA_CHECK(cudaStreamSynchronize(s_));  // the task lists are reused
        }
        d_scr.release();
        d_tscr.release();

        // collapse: occupied levels = set bits of the chunk count, lowest first
        std::vector<uint32_t> loff(nbf + 1, 0), list, bcap(nbf, 0);
        std::vector<unsigned long long> boff(nbf + 1, 0);
        for (uint32_t j = 0; j < nbf; j++) {
            const uint32_t C = nch[j];
            uint32_t levels = 0;
            for (uint32_t l = 0; (1ull << l) <= C; l++)
                if (C & (1u << l)) {
                    list.push_back(sbase[j] + ((C >> (l + 1)) << (l + 1)));
                    levels++;
                }
            loff[j + 1] = (uint32_t)list.size();
            bcap[j] = std::max<uint32_t>(levels, 1) * L;
            // two merge buffers of 3 arrays each, then (cap + 1) tied-prefix words
            boff[j + 1] = boff[j] + 6ull * bcap[j];
        }
        // tied-prefix offsets are boff[j] / 6 + j (cap + 1 words per feature)
        DevMem d_loff, d_list, d_boff, d_bcap, d_buf, d_tbuf, d_fin, d_cuts, d_ncuts;
        upload(d_loff, loff, s_);
        upload(d_list, list, s_);
        upload(d_boff, boff, s_);
        upload(d_bcap, bcap, s_);
        d_buf.alloc(boff[nbf] * 4);
        d_tbuf.alloc((boff[nbf] / 6 + nbf) * 4);
        d_fin.alloc((size_t)nbf * L * 12);
        d_cuts.alloc((size_t)nbf * max_bin * 4);
        d_ncuts.alloc((size_t)nbf * 4);
        count_launch();
        k_collapse_cuts<<<nbf, kSkThreads, 0, s_>>>(S, d_loff.as<uint32_t>(), d_list.as<uint32_t>(),
                                                    d_boff.as<unsigned long long>(), d_bcap.as<uint32_t>(),
                                                    d_buf.as<float>(), d_tbuf.as<uint32_t>(), d_fin.as<float>(),
                                                    max_bin, d_cuts.as<float>(), d_ncuts.as<uint32_t>());
        FB_CUDA_CHECK(cudaGetLastError());
        std::vector<float> hc((size_t)nbf * max_bin);
        std::vector<uint32_t> hn(nbf);
        FB_CUDA_CHECK(cudaMemcpyAsync(hc.data(), d_cuts.p, hc.size() * 4, cudaMemcpyDeviceToHost, s_));
        FB_CUDA_CHECK(cudaMemcpyAsync(hn.data(), d_ncuts.p, hn.size() * 4, cudaMemcpyDeviceToHost, s_));
        FB_CUDA_CHECK(cudaStreamSynchronize(s_));
        for (uint32_t j = 0; j < nbf; j++) {
            if (hn[j] > max_bin - 1) throw std::runtime_error("device sketch produced too many cuts");
            per[b0 + j].assign(hc.begin() + (size_t)j * max_bin, hc.begin() + (size_t)j * max_bin + hn[j]);
        }
    }
}

void DeviceMatrix::categorical_scan(const std::vector<uint32_t>& feats, std::vector<int32_t>& max_code,
                                    int64_t& bad_feat) {
    max_code.assign(feats.size(), -1);
    bad_feat = -1;
    if (feats.empty() || n_ == 0) return;
    DevMem d_feats, d_max, d_bad;
    upload(d_feats, feats, s_);
    upload(d_max, max_code, s_);
    d_bad.alloc(feats.size() * 4);
    FB_CUDA_CHECK(cudaMemsetAsync(d_bad.p, 0, feats.size() * 4, s_));
    const uint32_t gx = std::min<uint32_t>(ceil_div(n_, 256), 148u * 4u);
    dim3 grid(gx, (uint32_t)feats.size());
    count_launch();
    k_cat_scan<<<grid, 256, 0, s_>>>(x_, n_, rs_, cs_, d_feats.as<uint32_t>(), d_max.as<int>(), d_bad.as<unsigned int>());
    FB_CUDA_CHECK(cudaGetLastError());
    std::vector<uint32_t> bad(feats.size());
    FB_CUDA_CHECK(cudaMemcpyAsync(max_code.data(), d_max.p, feats.size() * 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(bad.data(), d_bad.p, feats.size() * 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    for (size_t i = 0; i < feats.size(); i++)
        if (bad[i]) { bad_feat = (int64_t)i; break; }
}

bool DeviceMatrix::bin_block(const uint32_t* feats, uint32_t n_feats, uint32_t width, const float* d_cuts,
                             const uint32_t* d_offsets, const uint8_t* d_cat, uint8_t* dst, uint32_t stride) {
    if (n_feats == 0 || n_feats > 128 || (width == 2 && n_feats > 64)) throw InputError("invalid block shape");
    DevMem d_feats, d_res;
    upload(d_feats, std::vector<uint32_t>(feats, feats + n_feats), s_);
    d_res.alloc(4);
    FB_CUDA_CHECK(cudaMemsetAsync(d_res.p, 0, 4, s_));
    FB_CUDA_CHECK(cudaMemsetAsync(dst, 0, (size_t)n_ * stride + 16, s_));
    if (n_) {
        const uint32_t grid = std::min<uint32_t>(ceil_div(n_, 8), 148u * 16u);
        count_launch();
        if (width == 2)
            k_bin_block<2><<<grid, 256, 0, s_>>>(x_, n_, rs_, cs_, d_feats.as<uint32_t>(), n_feats, d_cuts, d_offsets, d_cat,
                                                 dst, stride, d_res.as<unsigned int>());
        else
            k_bin_block<1><<<grid, 256, 0, s_>>>(x_, n_, rs_, cs_, d_feats.as<uint32_t>(), n_feats, d_cuts, d_offsets, d_cat,
                                                 dst, stride, d_res.as<unsigned int>());
        FB_CUDA_CHECK(cudaGetLastError());
    }
    uint32_t res = 0;
    FB_CUDA_CHECK(cudaMemcpyAsync(&res, d_res.p, 4, cudaMemcpyDeviceToHost, s_));
    FB_CUDA_CHECK(cudaStreamSynchronize(s_));
    return res != 0;
}

}  // namespace fbg
