// TreeSHAP over root-to-leaf paths (sm_100a).
//
// The reference's QuadratureTreeSHAP (model/explain.rs:198-400) walks every
// node of a tree per row and divides at every edge.  Its result is, for each
// leaf L with value v and each feature f on the path to L (repeated splits
// on f merged into one element):
//
//     phi_f += v (o_f - z_f) sum_i w_i prod_{g != f} (z_g + (o_g - z_g) y_i)
//
// where z_g is the product of the cover ratios (branch_weight) of g's edges
// on the path, o_g is 1 when the row satisfies every one of g's conditions on
// the path and 0 otherwise, and (y_i, w_i) is the quadrature rule on [0, 1].
// The integrand is a polynomial of degree < k (k = features on the path), so
// any rule exact to that degree gives the reference's value; the reference's
// 8-point endpoint-squared rule is exact for k <= 8.  Models whose paths all
// have k <= 8 use a 4-point Gauss-Legendre rule (also exact); others use the
// reference's own rule, so both compute the same quadrature sum.  The result
// differs from the reference only by f32 rounding (the parity bar is 1e-5).
//
// Everything except o_g is independent of the row, so the host precomputes
// per path element and rule point a_o = z + (o - z) y (o = 0, 1), b_o = w / a_o
// and c_o = v (o - z).  Per row and path the device only tests the row
// against each element's condition (an interval [lo, hi), the NaN default
// direction, or a category mask), multiplies P_i = prod_g a_{o_g,i}, and adds
// c_{o_f} sum_i b_{o_f,i} P_i to phi_f: no division, no recursion, no
// per-thread stack.
//
// Layout: one thread per row; the CTA's rows keep x and an f32 partial of phi
// in shared memory ([feature][thread], conflict-free), and the path elements
// stream through shared memory in chunks of whole paths, read by every thread
// at the same address (broadcast).  Every kFlushChunks chunks (about one
// depth-8 tree's paths) each thread adds its rows' partials into f64 totals
// in a per-CTA global scratch block ([feature][thread], coalesced, resident
// in L2) and clears them: a partial sums at most one term per path, like the
// reference's per-tree f32 sums, and the totals over trees stay f64.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"

namespace fbg {

namespace {

constexpr int kPathThreads = 128;
constexpr uint32_t kChunkBytes = 16 * 1024;
constexpr uint32_t kFlushChunks = 8;

// Element record, in 32-bit words: [0] feature | flags << 24, [1] lo (f32) or
// category-mask index, [2] hi (f32), [3] elements in the path (first element
// of a path only), then a0[M], a1[M], b0[M], b1[M], c0, c1, z and a pad word.
constexpr uint32_t kElemNanOk = 1u, kElemCat = 2u, kElemOutOk = 4u;
template <int M> __host__ __device__ constexpr uint32_t elem_words() { return 4 + 4 * M + 4; }

// Row test of one path element: every edge x < c (left) or x >= c (right),
// merged into lo <= x < hi (hi = NaN when no edge bounds it above); NaN rows
// follow the default directions; categorical rows test the intersection of
// the edges' category sets (data/categorical.rs:330-345).
__device__ __forceinline__ bool elem_test(uint4 h, float x, const uint32_t* __restrict__ cat_masks, uint32_t mw) {
    const uint32_t fl = h.x >> 24;
    if (x != x) return (fl & kElemNanOk) != 0;
    if (fl & kElemCat) {
        if (x < 0.0f || x >= 16777216.0f) return (fl & kElemOutOk) != 0;
        const uint32_t code = (uint32_t)x;
        return code < 32u * mw ? ((cat_masks[h.y * mw + (code >> 5)] >> (code & 31u)) & 1u) != 0
                               : (fl & kElemOutOk) != 0;
    }
    return !(x < __uint_as_float(h.y)) && !(x >= __uint_as_float(h.z));
}

template <int M>
__device__ __forceinline__ void load_vec(const uint32_t* p, float (&v)[M]) {
#pragma unroll
    for (int q = 0; q < M / 4; q++) {
        const float4 f = reinterpret_cast<const float4*>(p)[q];
        v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
}

// R rows per thread (rows t and t + kPathThreads of a CTA tile): the path
// data each element loads serves R independent product chains.
template <int M, int KMAX, int R>
__global__ void __launch_bounds__(kPathThreads) k_shap_paths(const float* __restrict__ X, uint64_t n, uint32_t F,
                                                             const uint4* __restrict__ elems,
                                                             const uint32_t* __restrict__ chunk_off,
                                                             uint32_t n_chunks, const uint32_t* __restrict__ cat_masks,
                                                             uint32_t mask_words, float bias, float root_mean,
                                                             double* __restrict__ acc, float* __restrict__ out) {
    constexpr uint32_t EW = elem_words<M>();
    constexpr uint32_t TR = kPathThreads * R;  // rows per CTA tile
    extern __shared__ __align__(16) uint32_t smem[];
    // a value receives one term per path that tests its feature (tens of
    // thousands per row): f32 partials over kFlushChunks chunks, f64 totals
    float* ph = reinterpret_cast<float*>(smem);                         // [F][TR]
    float* xs = ph + (size_t)F * TR;                                    // [F][TR]
    uint32_t* ch = reinterpret_cast<uint32_t*>(xs + (size_t)F * TR);    // chunk of elements
    double* tot = acc + (size_t)blockIdx.x * F * TR;                    // [F][TR] f64 totals
    const uint32_t t = threadIdx.x;
    for (uint64_t r0 = (uint64_t)blockIdx.x * TR; r0 < n; r0 += (uint64_t)gridDim.x * TR) {
        const uint32_t rows = (uint32_t)min((uint64_t)TR, n - r0);
        __syncthreads();
        for (uint32_t i = t; i < rows * F; i += kPathThreads) {
            const uint32_t rr = i / F, f = i - rr * F;
            xs[f * TR + rr] = X[r0 * F + i];
        }
        for (uint32_t i = t; i < F * TR; i += kPathThreads) ph[i] = 0.0f;
        bool flushed = false;  // uniform: the flushes follow the chunk count
        for (uint32_t c = 0; c < n_chunks; c++) {
            if (c > 0 && c % kFlushChunks == 0) {
                // each thread moves its own rows' partials (no other thread touches them)
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const uint32_t rr = t + r * kPathThreads;
                    if (rr < rows)
                        for (uint32_t f = 0; f < F; f++) {
                            float* p = ph + f * TR + rr;
                            double* q = tot + f * TR + rr;
                            *q = flushed ? __dadd_rn(*q, (double)*p) : (double)*p;
                            *p = 0.0f;
                        }
                }
                flushed = true;
            }
            const uint32_t e0 = chunk_off[c], e1 = chunk_off[c + 1];
            __syncthreads();
            const uint4* src = elems + (size_t)e0 * (EW / 4);
            uint4* dst = reinterpret_cast<uint4*>(ch);
            for (uint32_t i = t; i < (e1 - e0) * (EW / 4); i += kPathThreads) dst[i] = src[i];
            __syncthreads();
            if (t >= rows) continue;
            uint32_t e = 0;
            while (e < e1 - e0) {
                const uint32_t k = ch[e * EW + 3];
                float P[R][M];
#pragma unroll
                for (int r = 0; r < R; r++)
#pragma unroll
                    for (int i = 0; i < M; i++) P[r][i] = 1.0f;
                uint32_t obits[R], feats[KMAX];
#pragma unroll
                for (int r = 0; r < R; r++) obits[r] = 0;
#pragma unroll
                for (int j = 0; j < KMAX; j++) {
                    if ((uint32_t)j < k) {
                        const uint32_t* E = ch + (e + j) * EW;
                        const uint4 h = *reinterpret_cast<const uint4*>(E);
                        const uint32_t f = h.x & 0xffffffu;
                        feats[j] = f;
                        float a0[M], a1[M];
                        load_vec<M>(E + 4, a0);
                        load_vec<M>(E + 4 + M, a1);
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            const bool o = elem_test(h, xs[f * TR + t + r * kPathThreads], cat_masks, mask_words);
                            obits[r] |= (o ? 1u : 0u) << j;
#pragma unroll
                            for (int i = 0; i < M; i++) P[r][i] = __fmul_rn(P[r][i], o ? a1[i] : a0[i]);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < KMAX; j++) {
                    if ((uint32_t)j < k) {
                        const uint32_t* E = ch + (e + j) * EW;
                        float b0[M], b1[M];
                        load_vec<M>(E + 4 + 2 * M, b0);
                        load_vec<M>(E + 4 + 3 * M, b1);
                        const float2 cc = *reinterpret_cast<const float2*>(E + 4 + 4 * M);
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            const bool o = (obits[r] >> j) & 1u;
                            float sacc = 0.0f;
#pragma unroll
                            for (int i = 0; i < M; i++) sacc = __fmaf_rn(o ? b1[i] : b0[i], P[r][i], sacc);
                            float* p = ph + feats[j] * TR + t + r * kPathThreads;
                            *p = __fadd_rn(*p, __fmul_rn(o ? cc.y : cc.x, sacc));
                        }
                    }
                }
                e += k;
            }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint32_t rr = t + r * kPathThreads;
            if (rr < rows) {
                float* o = out + (r0 + rr) * (uint64_t)(F + 1);
                for (uint32_t f = 0; f < F; f++) {
                    const double v = (double)ph[f * TR + rr];
                    o[f] = __double2float_rn(flushed ? __dadd_rn(tot[f * TR + rr], v) : v);
                }
                o[F] = __fadd_rn(__fadd_rn(0.0f, root_mean), bias);  // explain.rs:725-726
            }
        }
    }
}

// SHAP interaction values (explain.rs:267-301, 762-805) over the same paths.
// For features i != j on a path the reference accumulates, at the deeper of
// the two edges, v (o_i - z_i)(o_j - z_j) sum_k w_k prod_{g != i,j} a_{g,k},
// and halves it when it symmetrises the matrix; the diagonal is the SHAP
// value minus the row's off-diagonal sum.  Here every pair of a path adds
// half that product to both (i, j) and (j, i), with
// w prod_{g != i,j} a_g = P b_i b_j / w (b = w / a).  One warp per row: lane j
// holds the path's element j, the warp multiplies P across lanes, and lane j
// adds its feature's SHAP term and its pairs with later elements.  The matrix
// accumulates in f64 in shared memory.
constexpr int kInterWarps = 4;
__host__ __device__ constexpr size_t inter_off(size_t bytes) { return (bytes + 15) & ~(size_t)15; }

template <int M>
__global__ void __launch_bounds__(kInterWarps * 32) k_shap_inter(const float* __restrict__ X, uint64_t n, uint32_t F,
                                                                 const uint4* __restrict__ elems,
                                                                 const uint32_t* __restrict__ chunk_off,
                                                                 uint32_t n_chunks,
                                                                 const uint32_t* __restrict__ cat_masks,
                                                                 uint32_t mask_words,
                                                                 const float* __restrict__ rule_w, uint32_t warps,
                                                                 float bias, float root_mean, float* __restrict__ out) {
    constexpr uint32_t EW = elem_words<M>();
    extern __shared__ __align__(16) uint32_t smem[];
    const uint32_t nc = F + 1;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const size_t mat = (size_t)nc * nc;
    // regions rounded to 16 bytes: matrices, diagonals, rows, path chunk
    uint8_t* base = reinterpret_cast<uint8_t*>(smem);
    double* mats = reinterpret_cast<double*>(base);                                  // [warps][nc][nc]
    double* diags = reinterpret_cast<double*>(base + inter_off(warps * mat * 8));    // [warps][nc]
    float* xs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(diags) + inter_off(warps * nc * 8));  // [warps][F]
    uint32_t* ch = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(xs) + inter_off((size_t)warps * F * 4));
    double* m = mats + warp * mat;
    double* dg = diags + warp * nc;
    float* x = xs + warp * F;
    float inv_w[M];
#pragma unroll
    for (int i = 0; i < M; i++) inv_w[i] = 1.0f / rule_w[i];
    for (uint64_t g0 = (uint64_t)blockIdx.x * warps; g0 < n; g0 += (uint64_t)gridDim.x * warps) {
        const uint64_t r = g0 + warp;
        const bool live = warp < warps && r < n;
        __syncthreads();
        if (live) {
            for (uint32_t i = lane; i < mat; i += 32) m[i] = 0.0;
            for (uint32_t i = lane; i < nc; i += 32) dg[i] = 0.0;
            for (uint32_t i = lane; i < F; i += 32) x[i] = X[r * F + i];
        }
        for (uint32_t c = 0; c < n_chunks; c++) {
            const uint32_t e0 = chunk_off[c], e1 = chunk_off[c + 1];
            __syncthreads();
            const uint4* src = elems + (size_t)e0 * (EW / 4);
            uint4* dst = reinterpret_cast<uint4*>(ch);
            for (uint32_t i = threadIdx.x; i < (e1 - e0) * (EW / 4); i += blockDim.x) dst[i] = src[i];
            __syncthreads();
            if (!live) continue;
            uint32_t e = 0;
            while (e < e1 - e0) {
                const uint32_t k = ch[e * EW + 3];
                const bool mine = lane < k;
                const uint32_t* E = ch + (e + (mine ? lane : 0)) * EW;
                const uint4 h = *reinterpret_cast<const uint4*>(E);
                const uint32_t f = h.x & 0xffffffu;
                const bool o = mine && elem_test(h, x[f], cat_masks, mask_words);
                float a[M], b[M], P[M];
                load_vec<M>(E + 4 + (o ? M : 0), a);
                load_vec<M>(E + 4 + 2 * M + (o ? M : 0), b);
                const float cj = __uint_as_float(E[4 + 4 * M + (o ? 1 : 0)]);
                const float dj = __fsub_rn(o ? 1.0f : 0.0f, __uint_as_float(E[4 + 4 * M + 2]));
#pragma unroll
                for (int i = 0; i < M; i++) P[i] = mine ? a[i] : 1.0f;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int i = 0; i < M; i++) P[i] = __fmul_rn(P[i], __shfl_xor_sync(0xffffffffu, P[i], off));
                if (mine) {
                    float s = 0.0f;
#pragma unroll
                    for (int i = 0; i < M; i++) s = __fmaf_rn(b[i], P[i], s);
                    dg[f] = __dadd_rn(dg[f], (double)__fmul_rn(cj, s));
                }
                for (uint32_t l = 1; l < k; l++) {
                    float bl[M];
#pragma unroll
                    for (int i = 0; i < M; i++) bl[i] = __shfl_sync(0xffffffffu, b[i], l);
                    const float dl = __shfl_sync(0xffffffffu, dj, l);
                    const uint32_t fl = __shfl_sync(0xffffffffu, f, l);
                    if (lane < l) {
                        float s = 0.0f;
#pragma unroll
                        for (int i = 0; i < M; i++) s = __fmaf_rn(__fmul_rn(b[i], bl[i]), __fmul_rn(P[i], inv_w[i]), s);
                        const double t = 0.5 * (double)cj * (double)dl * (double)s;
                        m[(size_t)f * nc + fl] = __dadd_rn(m[(size_t)f * nc + fl], t);
                        m[(size_t)fl * nc + f] = __dadd_rn(m[(size_t)fl * nc + f], t);
                    }
                }
                __syncwarp();  // the next path's lanes may update the same entries
                e += k;
            }
        }
        __syncwarp();
        if (live) {
            // diagonal: the additive value minus the row's interactions
            for (uint32_t i = lane; i < nc; i += 32) {
                double v = i == F ? (double)__fadd_rn(__fadd_rn(0.0f, root_mean), bias) : dg[i];
                for (uint32_t j = 0; j < nc; j++)
                    if (j != i) v -= m[(size_t)i * nc + j];
                m[(size_t)i * nc + i] = v;
            }
            __syncwarp();
            float* o = out + r * mat;
            for (uint32_t i = lane; i < mat; i += 32) o[i] = __double2float_rn(m[i]);
        }
    }
}

// Interaction values of models with too many features for a shared-memory
// matrix ((F+1)^2 f64 per row): the arithmetic of k_shap_inter, one warp (one
// CTA) per row of a batch, the row's off-diagonal sums ([nc][nc]) and SHAP
// values ([nc]) in global f64 scratch zeroed by the caller; k_inter_finish
// then forms the diagonal and writes the f32 matrix.  Within a path no entry
// is updated twice, and __syncwarp orders one path's updates before the
// next's.
template <int M>
__global__ void __launch_bounds__(32) k_shap_inter_global(const float* __restrict__ X, uint64_t r0, uint32_t rows,
                                                          uint32_t F, const uint4* __restrict__ elems,
                                                          const uint32_t* __restrict__ chunk_off, uint32_t n_chunks,
                                                          const uint32_t* __restrict__ cat_masks, uint32_t mask_words,
                                                          const float* __restrict__ rule_w, double* __restrict__ scratch) {
    constexpr uint32_t EW = elem_words<M>();
    extern __shared__ __align__(16) uint32_t smem[];
    const uint32_t nc = F + 1, lane = threadIdx.x;
    const size_t mat = (size_t)nc * nc;
    float* x = reinterpret_cast<float*>(smem);                   // [F]
    uint32_t* ch = smem + ((F + 3u) & ~3u);                      // path chunk (16-byte aligned)
    float inv_w[M];
#pragma unroll
    for (int i = 0; i < M; i++) inv_w[i] = 1.0f / rule_w[i];
    for (uint32_t rr = blockIdx.x; rr < rows; rr += gridDim.x) {
        const uint64_t r = r0 + rr;
        double* m = scratch + (size_t)rr * (mat + nc);
        double* dg = m + mat;
        __syncwarp();
        for (uint32_t i = lane; i < F; i += 32) x[i] = X[r * F + i];
        for (uint32_t c = 0; c < n_chunks; c++) {
            const uint32_t e0 = chunk_off[c], e1 = chunk_off[c + 1];
            __syncwarp();
            const uint4* src = elems + (size_t)e0 * (EW / 4);
            uint4* dst = reinterpret_cast<uint4*>(ch);
            for (uint32_t i = lane; i < (e1 - e0) * (EW / 4); i += 32) dst[i] = src[i];
            __syncwarp();
            uint32_t e = 0;
            while (e < e1 - e0) {
                const uint32_t k = ch[e * EW + 3];
                const bool mine = lane < k;
                const uint32_t* E = ch + (e + (mine ? lane : 0)) * EW;
                const uint4 h = *reinterpret_cast<const uint4*>(E);
                const uint32_t f = h.x & 0xffffffu;
                const bool o = mine && elem_test(h, x[f], cat_masks, mask_words);
                float a[M], b[M], P[M];
                load_vec<M>(E + 4 + (o ? M : 0), a);
                load_vec<M>(E + 4 + 2 * M + (o ? M : 0), b);
                const float cj = __uint_as_float(E[4 + 4 * M + (o ? 1 : 0)]);
                const float dj = __fsub_rn(o ? 1.0f : 0.0f, __uint_as_float(E[4 + 4 * M + 2]));
#pragma unroll
                for (int i = 0; i < M; i++) P[i] = mine ? a[i] : 1.0f;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int i = 0; i < M; i++) P[i] = __fmul_rn(P[i], __shfl_xor_sync(0xffffffffu, P[i], off));
                if (mine) {
                    float sacc = 0.0f;
#pragma unroll
                    for (int i = 0; i < M; i++) sacc = __fmaf_rn(b[i], P[i], sacc);
                    dg[f] = __dadd_rn(dg[f], (double)__fmul_rn(cj, sacc));
                }
                for (uint32_t l = 1; l < k; l++) {
                    float bl[M];
#pragma unroll
                    for (int i = 0; i < M; i++) bl[i] = __shfl_sync(0xffffffffu, b[i], l);
                    const float dl = __shfl_sync(0xffffffffu, dj, l);
                    const uint32_t fl = __shfl_sync(0xffffffffu, f, l);
                    if (lane < l) {
                        float sacc = 0.0f;
#pragma unroll
                        for (int i = 0; i < M; i++)
                            sacc = __fmaf_rn(__fmul_rn(b[i], bl[i]), __fmul_rn(P[i], inv_w[i]), sacc);
                        const double t = 0.5 * (double)cj * (double)dl * (double)sacc;
                        m[(size_t)f * nc + fl] = __dadd_rn(m[(size_t)f * nc + fl], t);
                        m[(size_t)fl * nc + f] = __dadd_rn(m[(size_t)fl * nc + f], t);
                    }
                }
                __syncwarp();
                e += k;
            }
        }
    }
}

// Diagonal (the SHAP value minus the row's interactions; the bias row takes
// the bias) and f32 output of k_shap_inter_global's rows: a warp per matrix
// row.
__global__ void __launch_bounds__(256) k_inter_finish(uint64_t r0, uint32_t rows, uint32_t F, float bias,
                                                      float root_mean, const double* __restrict__ scratch,
                                                      float* __restrict__ out) {
    const uint32_t nc = F + 1, lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const size_t mat = (size_t)nc * nc;
    const uint64_t total = (uint64_t)rows * nc;
    for (uint64_t g = (uint64_t)blockIdx.x * 8 + warp; g < total; g += (uint64_t)gridDim.x * 8) {
        const uint32_t rr = (uint32_t)(g / nc), i = (uint32_t)(g % nc);
        const double* m = scratch + (size_t)rr * (mat + nc);
        const double* mi = m + (size_t)i * nc;
        float* o = out + (r0 + rr) * mat + (size_t)i * nc;
        double off = 0.0;
        for (uint32_t j = lane; j < nc; j += 32) {
            const double v = mi[j];
            if (j != i) {
                off += v;
                o[j] = __double2float_rn(v);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) off += __shfl_xor_sync(0xffffffffu, off, d);
        if (lane == 0) {
            const double base = i == F ? (double)__fadd_rn(__fadd_rn(0.0f, root_mean), bias) : m[mat + i];
            o[i] = __double2float_rn(base - off);
        }
    }
}

}  // namespace

// Gauss-Legendre rule with m points on [0, 1] (Golub-Welsch-free Newton on
// the Legendre recurrence, f64).
static void gauss_legendre01(int m, double* y, double* w) {
    for (int i = 0; i < m; i++) {
        double x = std::cos(3.14159265358979323846 * (i + 0.75) / (m + 0.5));
        double dp = 1.0;
        for (int it = 0; it < 100; it++) {
            double p0 = 1.0, p1 = x;
            for (int k = 2; k <= m; k++) {
                const double pk = ((2.0 * k - 1.0) * x * p1 - (k - 1.0) * p0) / k;
                p0 = p1;
                p1 = pk;
            }
            dp = m * (x * p1 - p0) / (x * x - 1.0);
            const double dx = p1 / dp;
            x -= dx;
            if (std::fabs(dx) < 1e-16) break;
        }
        y[i] = 0.5 * (x + 1.0);
        w[i] = 1.0 / ((1.0 - x * x) * dp * dp);  // (2 / ((1 - x^2) P'^2)) / 2
    }
}

void ShapPaths::build(const std::vector<DevNode>& nodes, const uint32_t* tree_off, uint32_t n_trees, uint32_t F,
                      const std::vector<uint32_t>& cat_off, const std::vector<uint32_t>& cat_len,
                      const uint32_t* cat_words, const float* rule_nodes, const float* rule_weights) {
    struct El {
        uint32_t feat;
        double z;
        float lo, hi;
        bool nan_ok, cat, out_ok;
        std::vector<uint32_t> mask;  // categorical: codes the row may hold (mask_words words)
    };
    struct Path {
        float v;
        std::vector<El> els;
    };
    supported = true;
    // words of a category mask: every set of the model fits (a bit per code)
    mask_words = 8;
    for (uint32_t t = 0; t < n_trees; t++)
        for (uint32_t i = tree_off[t]; i < tree_off[t + 1]; i++)
            if ((nodes[i].meta >> 24) & kNodeCategorical) mask_words = std::max(mask_words, cat_len[i]);
    std::vector<Path> paths;
    std::vector<int> pos(F, -1);
    std::vector<El> st;
    uint32_t kmax = 0;
    for (uint32_t t = 0; t < n_trees; t++) {
        const uint32_t a = tree_off[t];
        const DevNode* nd = nodes.data() + a;
        if ((nd[0].meta >> 24) & kNodeLeaf) continue;  // explain.rs:393-400: a leaf root adds nothing
        // explicit DFS: (node, next child to visit, undo record)
        struct Fr {
            uint32_t i;
            int stage;
            int slot;
            El saved;
            bool fresh;
        };
        std::vector<Fr> stack;
        stack.push_back(Fr{0, 0, -1, El{}, false});
        while (!stack.empty()) {
            Fr& fr = stack.back();
            const DevNode& d = nd[fr.i];
            if ((d.meta >> 24) & kNodeLeaf) {
                paths.push_back(Path{d.val, st});
                kmax = std::max<uint32_t>(kmax, (uint32_t)st.size());
                stack.pop_back();
                continue;
            }
            // undo the previous child's edge
            if (fr.stage > 0 && fr.slot >= 0) {
                if (fr.fresh) {
                    pos[st.back().feat] = -1;
                    st.pop_back();
                } else {
                    st[fr.slot] = fr.saved;
                }
            }
            if (fr.stage == 2) {
                stack.pop_back();
                continue;
            }
            const bool left = fr.stage == 0;
            const uint32_t child = (uint32_t)(left ? d.left : d.right);
            fr.stage++;
            const uint32_t f = d.meta & 0xffffffu;
            const uint32_t flags = d.meta >> 24;
            // explain.rs:182-192 branch_weight in f32
            float cw;
            const float pc = d.hess, cc = nd[child].hess;
            if (pc <= 0.0f) {
                cw = 0.5f;
            } else {
                cw = cc / pc;
                if (cw < 1e-12f) cw = 1e-12f;
            }
            int slot = pos[f];
            fr.fresh = slot < 0;
            if (fr.fresh) {
                El e{};
                e.feat = f;
                e.z = 1.0;
                e.lo = -INFINITY;
                e.hi = INFINITY;
                e.nan_ok = true;
                e.cat = (flags & kNodeCategorical) != 0;
                e.out_ok = true;
                e.mask.assign(mask_words, 0xffffffffu);
                st.push_back(e);
                slot = (int)st.size() - 1;
                pos[f] = slot;
            } else {
                fr.saved = st[slot];
            }
            fr.slot = slot;
            El& e = st[slot];
            e.z *= (double)cw;
            e.nan_ok = e.nan_ok && (((flags & kNodeDefaultLeft) != 0) == left);
            if (flags & kNodeCategorical) {
                const uint32_t co = cat_off[a + fr.i], cl = cat_len[a + fr.i];
                for (uint32_t wi = 0; wi < mask_words; wi++) {
                    const uint32_t s = wi < cl ? cat_words[co + wi] : 0u;
                    e.mask[wi] &= left ? ~s : s;
                }
                e.out_ok = e.out_ok && left;
            } else if (left) {
                e.hi = std::min(e.hi, d.val);
            } else {
                e.lo = std::max(e.lo, d.val);
            }
            stack.push_back(Fr{child, 0, -1, El{}, false});
        }
    }
    // rule: 4-point Gauss-Legendre when every path has at most 8 features,
    // else the reference's 8-point endpoint-squared rule
    M = kmax <= 8 ? 4 : 8;
    KMAX = M == 4 ? 8 : 14;
    if (kmax > 14) {
        supported = false;
        return;
    }
    double y[8], w[8];
    if (M == 4) {
        gauss_legendre01(4, y, w);
    } else {
        for (int i = 0; i < 8; i++) { y[i] = rule_nodes[i]; w[i] = rule_weights[i]; }
    }
    for (int i = 0; i < 8; i++) rule_w8[i] = rule_weights[i];
    const uint32_t EW = 4 + 4 * M + 4;
    const uint32_t chunk_elems = kChunkBytes / (EW * 4);
    words.clear();
    masks.clear();
    chunk_off.assign(1, 0);
    uint32_t in_chunk = 0, total = 0;
    auto clamp = [](double x) {
        if (!(x == x)) return 0.0f;
        if (x > FLT_MAX) return FLT_MAX;
        if (x < -FLT_MAX) return -FLT_MAX;
        return (float)x;
    };
    for (const Path& p : paths) {
        const uint32_t k = (uint32_t)p.els.size();
        if (in_chunk + k > chunk_elems) {
            chunk_off.push_back(total);
            in_chunk = 0;
        }
        for (uint32_t j = 0; j < k; j++) {
            const El& e = p.els[j];
            uint32_t rec[4 + 4 * 8 + 4] = {};
            const uint32_t fl = (e.nan_ok ? kElemNanOk : 0u) | (e.cat ? kElemCat : 0u) | (e.out_ok ? kElemOutOk : 0u);
            rec[0] = (e.feat & 0xffffffu) | (fl << 24);
            if (e.cat) {
                rec[1] = (uint32_t)(masks.size() / mask_words);
                masks.insert(masks.end(), e.mask.begin(), e.mask.end());
                rec[2] = 0;
            } else {
                // no upper bound: hi = NaN, so the test !(x >= hi) always passes (x = +inf included)
                const float hi = e.hi == INFINITY ? NAN : e.hi;
                std::memcpy(&rec[1], &e.lo, 4);
                std::memcpy(&rec[2], &hi, 4);
            }
            rec[3] = j == 0 ? k : 0u;
            float* tab = reinterpret_cast<float*>(rec + 4);
            for (int i = 0; i < M; i++) {
                const double a0 = e.z * (1.0 - y[i]), a1 = e.z + (1.0 - e.z) * y[i];
                tab[i] = clamp(a0);
                tab[M + i] = clamp(a1);
                tab[2 * M + i] = clamp(w[i] / a0);
                tab[3 * M + i] = clamp(w[i] / a1);
            }
            tab[4 * M] = clamp((double)p.v * (0.0 - e.z));
            tab[4 * M + 1] = clamp((double)p.v * (1.0 - e.z));
            tab[4 * M + 2] = (float)e.z;  // interactions: o - z of a partner
            words.insert(words.end(), rec, rec + EW);
        }
        in_chunk += k;
        total += k;
    }
    chunk_off.push_back(total);
    if (chunk_off.size() >= 2 && chunk_off[chunk_off.size() - 2] == total) chunk_off.pop_back();
    n_elems = total;
}

void ShapPaths::upload(cudaStream_t s) {
    d_words.alloc(std::max<size_t>(words.size(), 4) * 4);
    d_chunks.alloc(chunk_off.size() * 4);
    d_masks.alloc(std::max<size_t>(masks.size(), mask_words) * 4);
    if (!words.empty())
        FB_CUDA_CHECK(cudaMemcpyAsync(d_words.p, words.data(), words.size() * 4, cudaMemcpyHostToDevice, s));
    FB_CUDA_CHECK(cudaMemcpyAsync(d_chunks.p, chunk_off.data(), chunk_off.size() * 4, cudaMemcpyHostToDevice, s));
    if (!masks.empty())
        FB_CUDA_CHECK(cudaMemcpyAsync(d_masks.p, masks.data(), masks.size() * 4, cudaMemcpyHostToDevice, s));
}


size_t ShapPaths::inter_smem_bytes(uint32_t F, uint32_t warps) {
    const size_t nc = F + 1;
    return inter_off(warps * nc * nc * 8) + inter_off(warps * nc * 8) + inter_off((size_t)warps * F * 4) + kChunkBytes;
}

uint32_t ShapPaths::inter_warps(uint32_t F) {
    for (uint32_t w = kInterWarps; w >= 1; w--)
        if (inter_smem_bytes(F, w) <= 200 * 1024) return w;
    return 0;
}

void ShapPaths::launch_inter(const float* X, uint64_t n, uint32_t F, float bias, float root_mean, float* out,
                             cudaStream_t s) {
    if (n == 0) return;
    const uint32_t warps = inter_warps(F);
    if (!d_rule_w.p) {
        double y[8], w[8];
        float wf[8];
        if (M == 4) gauss_legendre01(4, y, w);
        for (int i = 0; i < M; i++) wf[i] = M == 4 ? (float)w[i] : rule_w8[i];
        d_rule_w.alloc(sizeof(float) * 8);
        FB_CUDA_CHECK(cudaMemcpyAsync(d_rule_w.p, wf, sizeof(float) * M, cudaMemcpyHostToDevice, s));
    }
    const uint32_t n_chunks = (uint32_t)chunk_off.size() - 1;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (warps == 0) {
        // the matrix does not fit shared memory: global f64 scratch, rows in
        // batches of at most 1 GiB of scratch
        const size_t nc = (size_t)F + 1;
        const size_t per_row = (nc * nc + nc) * 8;
        const size_t gsmem = (size_t)((F + 3u) & ~3u) * 4 + kChunkBytes;
        if (gsmem > 227 * 1024) throw InputError("pred_interactions on the device supports at most 51000 features");
        const uint64_t R = std::max<uint64_t>(1, std::min<uint64_t>(n, (1ull << 30) / per_row));
        if (d_inter_scratch.bytes < R * per_row) d_inter_scratch.alloc(R * per_row);
        double* scr = d_inter_scratch.as<double>();
        for (uint64_t r0 = 0; r0 < n; r0 += R) {
            const uint32_t rows = (uint32_t)std::min<uint64_t>(R, n - r0);
            FB_CUDA_CHECK(cudaMemsetAsync(scr, 0, rows * per_row, s));
#define FB_SG(MM)                                                                                                  \
    do {                                                                                                           \
        cudaFuncSetAttribute(k_shap_inter_global<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsmem);    \
        count_launch();                                                                                            \
        k_shap_inter_global<MM><<<rows, 32, gsmem, s>>>(X, r0, rows, F, d_words.as<uint4>(), d_chunks.as<uint32_t>(), \
                                                        n_chunks, d_masks.as<uint32_t>(), mask_words,              \
                                                        d_rule_w.as<float>(), scr);                                \
    } while (0)
            if (M == 4) FB_SG(4);
            else FB_SG(8);
#undef FB_SG
            const uint64_t warps_total = (uint64_t)rows * nc;
            const uint32_t grid = (uint32_t)std::min<uint64_t>((warps_total + 7) / 8, (uint64_t)sms * 8);
            count_launch();
            k_inter_finish<<<grid, 256, 0, s>>>(r0, rows, F, bias, root_mean, scr, out);
        }
        return;
    }
    const size_t smem = inter_smem_bytes(F, warps);
    const uint64_t groups = (n + warps - 1) / warps;
#define FB_SI(MM)                                                                                                  \
    do {                                                                                                           \
        cudaFuncSetAttribute(k_shap_inter<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);            \
        int per_sm = 1;                                                                                            \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_shap_inter<MM>, kInterWarps * 32, smem);          \
        const uint64_t grid = std::min<uint64_t>(groups, (uint64_t)sms * std::max(per_sm, 1));                     \
        count_launch();                                                                                            \
        k_shap_inter<MM><<<(unsigned)grid, kInterWarps * 32, smem, s>>>(                                          \
            X, n, F, d_words.as<uint4>(), d_chunks.as<uint32_t>(), n_chunks, d_masks.as<uint32_t>(), mask_words,   \
            d_rule_w.as<float>(), warps, bias, root_mean, out);                                                    \
    } while (0)
    if (M == 4) FB_SI(4);
    else FB_SI(8);
#undef FB_SI
}

// two rows per thread: the path data read from shared memory serves two product chains
constexpr int kPathRows = 2;

size_t ShapPaths::smem_bytes(uint32_t F) { return (size_t)F * kPathThreads * kPathRows * (4 + 4) + kChunkBytes; }

void ShapPaths::launch(const float* X, uint64_t n, uint32_t F, float bias, float root_mean, float* out,
                       cudaStream_t s) const {
    if (n == 0) return;
    const uint32_t n_chunks = (uint32_t)chunk_off.size() - 1;
    const size_t smem = smem_bytes(F);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int R = kPathRows;
    const uint64_t tiles = (n + (uint64_t)kPathThreads * R - 1) / ((uint64_t)kPathThreads * R);
#define FB_SP(MM, KK, RR)                                                                                            \
    do {                                                                                                             \
        cudaFuncSetAttribute(k_shap_paths<MM, KK, RR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);      \
        int per_sm = 1;                                                                                              \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_shap_paths<MM, KK, RR>, kPathThreads, smem);        \
        const uint64_t grid = std::min<uint64_t>(tiles, (uint64_t)sms * std::max(per_sm, 1));                        \
        const size_t acc_bytes = grid * F * (size_t)kPathThreads * RR * 8;                                           \
        if (d_acc.bytes < acc_bytes) d_acc.alloc(acc_bytes);                                                         \
        count_launch();                                                                                              \
        k_shap_paths<MM, KK, RR><<<(unsigned)grid, kPathThreads, smem, s>>>(                                        \
            X, n, F, d_words.as<uint4>(), d_chunks.as<uint32_t>(), n_chunks, d_masks.as<uint32_t>(), mask_words,    \
            bias, root_mean, d_acc.as<double>(), out);                                                               \
    } while (0)
    if (M == 4) FB_SP(4, 8, kPathRows);
    else FB_SP(8, 14, kPathRows);
#undef FB_SP
}

}  // namespace fbg
