// Training kernels (sm_100a).  See train_kernels.cuh for the level pipeline.
#include <cfloat>

#include "train_kernels.cuh"

namespace fbg {

// The pair of (accumulate slot, packed bin index) in a level's accumulate
// histograms.  Unsharded, slot * slot_pairs + bin.  For the feature-sharded
// split search of a row-sharded run the histograms are laid out rank-major,
// [rank][accumulate slot][that rank's features' bins], so one reduce-scatter
// hands each rank the sums of its own features; a feature's packed index
// carries its rank in the top 8 bits and rank_stride (TreeState) is the size
// of a rank's block.
__device__ __forceinline__ Pair* acc_bin(Pair* hist_acc, uint32_t acc_slot, unsigned long long slot_pairs,
                                         unsigned long long rank_stride, uint32_t packed) {
    return hist_acc + (unsigned long long)(packed >> 24) * rank_stride + (unsigned long long)acc_slot * slot_pairs +
           (packed & 0xffffffu);
}

// ------------------------------------------------------------------ scans
template <int NT>
__device__ __forceinline__ Pair block_excl_scan_pair(Pair v, Pair* warp_tot, Pair& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Pair incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Pair t{__shfl_up_sync(0xffffffffu, incl.g, o), __shfl_up_sync(0xffffffffu, incl.h, o)};
        if (lane >= o) incl = padd(incl, t);
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        Pair t = lane < NT / 32 ? warp_tot[lane] : Pair{0, 0};
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            Pair u{__shfl_up_sync(0xffffffffu, t.g, o), __shfl_up_sync(0xffffffffu, t.h, o)};
            if (lane >= o) t = padd(t, u);
        }
        if (lane < NT / 32) warp_tot[lane] = t;
    }
    __syncthreads();
    Pair base = warp > 0 ? warp_tot[warp - 1] : Pair{0, 0};
    total = warp_tot[NT / 32 - 1];
    __syncthreads();
    return psub(padd(base, incl), v);
}

template <int NT>
__device__ __forceinline__ uint32_t block_excl_scan_u32(uint32_t v, uint32_t* warp_tot, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t t = lane < NT / 32 ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        if (lane < NT / 32) warp_tot[lane] = t;
    }
    __syncthreads();
    uint32_t base = warp > 0 ? warp_tot[warp - 1] : 0u;
    total = warp_tot[NT / 32 - 1];
    __syncthreads();
    return base + incl - v;
}

template <int NT>
__device__ __forceinline__ unsigned long long block_excl_scan_u64(unsigned long long v, unsigned long long* warp_tot,
                                                                  unsigned long long& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        unsigned long long t = lane < NT / 32 ? warp_tot[lane] : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            unsigned long long u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        if (lane < NT / 32) warp_tot[lane] = t;
    }
    __syncthreads();
    unsigned long long base = warp > 0 ? warp_tot[warp - 1] : 0ull;
    total = warp_tot[NT / 32 - 1];
    __syncthreads();
    return base + incl - v;
}

// Largest j in [0, n) with prefix[j] <= x (prefix ascending, prefix[0] <= x).
template <class T>
__device__ __forceinline__ uint32_t find_segment(const T* prefix, uint32_t n, T x) {
    uint32_t lo = 0, hi = n;  // invariant: prefix[lo] <= x, answer in [lo, hi)
    while (hi - lo > 1) {
        uint32_t mid = (lo + hi) >> 1;
        if (prefix[mid] <= x) lo = mid; else hi = mid;
    }
    return lo;
}

// find_segment by a whole warp: each round the 32 lanes probe 32 evenly
// spaced entries at once and a ballot keeps the last one <= x, so a table of
// up to 1024 entries takes two dependent loads instead of log2(n).  Every lane
// of the warp calls it and gets the same answer.
template <class T>
__device__ __forceinline__ uint32_t find_segment_warp(const T* prefix, uint32_t n, T x) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t lo = 0, hi = n;  // invariant: prefix[lo] <= x, answer in [lo, hi)
    while (hi - lo > 1) {
        const uint32_t step = (hi - lo + 31u) / 32u;
        const uint32_t i = lo + lane * step;
        const bool le = i < hi && prefix[i] <= x;
        const uint32_t mask = __ballot_sync(0xffffffffu, le);
        const uint32_t last = 31u - (uint32_t)__clz(mask);  // lane 0 always holds (prefix[lo] <= x)
        lo = lo + last * step;
        hi = min(hi, lo + step);
    }
    return lo;
}

// ------------------------------------------------------------------ gradients
// data/subsample.rs:45-78 row hash (SplitMix64 finalizer of seed, tree, row).
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ bool row_selected(unsigned long long row, unsigned long long th,
                                             unsigned long long seed, unsigned long long tree) {
    if (th == ~0ull) return true;
    unsigned long long t = tree * 0x9E3779B97F4A7C15ull;
    unsigned long long h = mix64(seed ^ ((t << 23) | (t >> 41)) ^ (row * 0xD6E8FEB86659FD93ull));
    return (h >> 11) < th;
}



__device__ __forceinline__ double bound_of(float v) {
    return isfinite(v) ? fabs((double)v) : __longlong_as_double(0x7ff0000000000000ll);
}

// Block max of two non-negative doubles folded into global maxima.  Bit
// patterns of non-negative doubles order like the values, so an integer max
// is exact and order independent.
__device__ __forceinline__ void fold_max(double mg, double mh, unsigned long long* maxbits) {
    __shared__ unsigned long long smg[32], smh[32];
    unsigned long long a = (unsigned long long)__double_as_longlong(mg);
    unsigned long long b = (unsigned long long)__double_as_longlong(mh);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a = max(a, __shfl_down_sync(0xffffffffu, a, o));
        b = max(b, __shfl_down_sync(0xffffffffu, b, o));
    }
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { smg[warp] = a; smh[warp] = b; }
    __syncthreads();
    if (warp == 0) {
        int nw = (blockDim.x + 31) >> 5;
        a = lane < nw ? smg[lane] : 0ull;
        b = lane < nw ? smh[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            a = max(a, __shfl_down_sync(0xffffffffu, a, o));
            b = max(b, __shfl_down_sync(0xffffffffu, b, o));
        }
        if (lane == 0) { atomicMax(&maxbits[0], a); atomicMax(&maxbits[1], b); }
    }
}

__device__ __forceinline__ void fold_sum(Pair s, unsigned long long* sum) {
    __shared__ long long sg[32], sh[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s.g = (long long)((unsigned long long)s.g + (unsigned long long)__shfl_down_sync(0xffffffffu, s.g, o));
        s.h = (long long)((unsigned long long)s.h + (unsigned long long)__shfl_down_sync(0xffffffffu, s.h, o));
    }
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sg[warp] = s.g; sh[warp] = s.h; }
    __syncthreads();
    if (warp == 0) {
        int nw = (blockDim.x + 31) >> 5;
        Pair t{lane < nw ? sg[lane] : 0ll, lane < nw ? sh[lane] : 0ll};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            t.g = (long long)((unsigned long long)t.g + (unsigned long long)__shfl_down_sync(0xffffffffu, t.g, o));
            t.h = (long long)((unsigned long long)t.h + (unsigned long long)__shfl_down_sync(0xffffffffu, t.h, o));
        }
        if (lane == 0) {
            atomicAdd(&sum[0], (unsigned long long)t.g);
            atomicAdd(&sum[1], (unsigned long long)t.h);
        }
    }
}

// types.rs:334-337 quantize: round-half-away of v * 2^k (exact product).
__device__ __forceinline__ Pair to_fixed(float g, float h, double gs, double hs) {
    return {(long long)round(__dmul_rn((double)g, gs)), (long long)round(__dmul_rn((double)h, hs))};
}

// Reference exact path (backend upload_and_quantize_gpair_sampled): mask
// unsampled rows of the host f32 pairs and fold the bounds.
__global__ void k_mask_max(GradArgs a) {
    double mg = 0.0, mh = 0.0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += blockDim.x * gridDim.x) {
        float g = a.gpair_in[2ull * i], h = a.gpair_in[2ull * i + 1];
        if (!row_selected(a.row0 + i, a.sub_th, a.sub_seed, a.sub_tree)) { g = 0.0f; h = 0.0f; }
        a.gpair_f32[2ull * i] = g;
        a.gpair_f32[2ull * i + 1] = h;
        mg = fmax(mg, bound_of(g));
        mh = fmax(mh, bound_of(h));
    }
    fold_max(mg, mh, a.maxbits);
}

// objective.rs:37-39,513-526: the gradient of one row, in the reference's f32
// operation order.  Logistic takes e = expf(-pred): the host's glibc expf in
// exact mode (reproduced on the device); in fast mode fexp_core alone (fexp.h:
// an f64 evaluation rounded once to f32, which differs from glibc on about
// 0.004 % of the inputs, by one unit in the last place).
// `m` is the row's margin (read by squared error only).
__device__ __forceinline__ void row_gradient_m(const GradArgs& a, uint32_t i, float e, float m, float& g, float& h) {
    float y = a.label[i];
    if (a.objective == 1) {
        float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
        float hh = __fmul_rn(s, __fsub_rn(1.0f, s));
        g = __fsub_rn(s, y);
        h = hh < 1e-16f ? 1e-16f : hh;
    } else {
        g = __fsub_rn(m, y);
        h = 1.0f;
    }
    if (a.weight) {  // training/mod.rs:5498-5505 weighted
        float w = a.weight[i];
        g = __fmul_rn(g, w);
        h = __fmul_rn(h, w);
    }
    if (!row_selected(a.row0 + i, a.sub_th, a.sub_seed, a.sub_tree)) { g = 0.0f; h = 0.0f; }
}
__device__ __forceinline__ void row_gradient(const GradArgs& a, uint32_t i, float e, float& g, float& h) {
    row_gradient_m(a, i, e, a.objective == 1 ? 0.0f : a.pred[i], g, h);
}

// The host C library's expf on the device: fexp_core, except on the inputs the
// exception table lists (fexp.h).  The probe loop is bounded by the table's
// longest probe sequence.
__device__ __forceinline__ float host_expf(float x, const uint2* tab, uint32_t probes) {
    const uint32_t key = __float_as_uint(x);
    uint32_t slot = fbx::exp_slot(key);
    for (uint32_t i = 0; i < probes; i++) {
        const uint2 e = tab[slot];
        if (e.x == fbx::kEmptyKey) break;  // before the key test: kEmptyKey is also a NaN input
        if (e.x == key) return __uint_as_float(e.y);
        slot = (slot + 1) & (fbx::kExpTableSlots - 1);
    }
    return fbx::fexp_core(x);
}

// host_expf with its first probe already loaded (t = tab[exp_slot(key)]).
__device__ __forceinline__ float host_expf_from(float x, uint32_t key, uint2 t, const uint2* tab, uint32_t probes) {
    if (t.x == fbx::kEmptyKey) return fbx::fexp_core(x);
    if (t.x == key) return __uint_as_float(t.y);
    uint32_t slot = fbx::exp_slot(key);
    for (uint32_t i = 1; i < probes; i++) {
        slot = (slot + 1) & (fbx::kExpTableSlots - 1);
        const uint2 e = __ldg(&tab[slot]);
        if (e.x == fbx::kEmptyKey) break;
        if (e.x == key) return __uint_as_float(e.y);
    }
    return fbx::fexp_core(x);
}

__global__ void k_expf_emulate(const uint2* tab, uint32_t probes, uint32_t begin, uint32_t count, uint32_t* out) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += blockDim.x * gridDim.x)
        out[i] = __float_as_uint(host_expf(__uint_as_float(begin + i), tab, probes));
}

// Gradient pass that only folds bounds and stores the f32 pairs (exact
// squared error, exact logistic with the emulated host expf, fast mode).
// Each thread takes kGradRows rows a step (a grid stride apart, so every load
// is coalesced) and issues their margin loads, then their first probes of the
// exception table, before it needs any of them: the pass is bound by the
// latency of those two dependent loads, not by their bytes.
constexpr int kGradRows = 4;
__global__ void __launch_bounds__(256) k_gradient_max(GradArgs a, int mode) {
    double mg = 0.0, mh = 0.0;
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x, n = a.n;
    for (uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += kGradRows * stride) {
        float e[kGradRows];
#pragma unroll
        for (int k = 0; k < kGradRows; k++) e[k] = 0.0f;
        if (a.objective == 1) {
            float x[kGradRows];
#pragma unroll
            for (int k = 0; k < kGradRows; k++) {
                const uint64_t i = i0 + k * stride;
                x[k] = i < n ? -a.pred[i] : 0.0f;
            }
            if (mode == 2) {
                uint2 t[kGradRows];
#pragma unroll
                for (int k = 0; k < kGradRows; k++)
                    t[k] = __ldg(&a.exptab[fbx::exp_slot(__float_as_uint(x[k]))]);
#pragma unroll
                for (int k = 0; k < kGradRows; k++)
                    e[k] = host_expf_from(x[k], __float_as_uint(x[k]), t[k], a.exptab, a.exp_probes);
            } else {
#pragma unroll
                for (int k = 0; k < kGradRows; k++) {
                    const uint64_t i = i0 + k * stride;
                    e[k] = mode == 1 ? fbx::fexp_core(x[k]) : (i < n ? a.host_exp[i] : 0.0f);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kGradRows; k++) {
            const uint64_t i = i0 + k * stride;
            if (i < n) {
                float g, h;
                row_gradient(a, (uint32_t)i, e[k], g, h);
                reinterpret_cast<float2*>(a.gpair_f32)[i] = make_float2(g, h);
                mg = fmax(mg, bound_of(g));
                mh = fmax(mh, bound_of(h));
            }
        }
    }
    fold_max(mg, mh, a.maxbits);
}

// Exact logistic with host exp: gradients recomputed on the device from e in
// the same f32 order as the host, then quantized with the host's scales.
__global__ void k_gradient_quantize_exp(GradArgs a) {
    Pair s{0, 0};
    double gs = a.scales[0], hs = a.scales[1];
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += blockDim.x * gridDim.x) {
        float g, h;
        row_gradient(a, i, a.host_exp[i], g, h);
        Pair f = to_fixed(g, h, gs, hs);
        a.fixed[i] = f;
        s = padd(s, f);
    }
    fold_sum(s, a.sum);
}

// objective.rs:1175-1219 softmax_gradients, one thread per row, in the
// reference's f32 order: wmax from the smallest positive normal f32, the
// exps of (m_k - wmax) summed in f64, p = e / (f32)sum,
// h = max(((2 p)(1 - p)) w, 1e-16), the label's class takes p - 1, g = p w.
// KR > 0: K <= KR and each class's exp is kept in registers between the
// sum and the division; KR = 0: any K, the exp evaluated again (same value).
template <bool FAST, int KR>
__global__ void k_softmax_grad(GradArgs a, uint32_t K, float* __restrict__ out) {
    const size_t n = a.n;
    auto ex = [&](float x) { return FAST ? fbx::fexp_core(x) : host_expf(x, a.exptab, a.exp_probes); };
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += blockDim.x * gridDim.x) {
        float wmax = FLT_MIN;
        for (uint32_t k = 0; k < K; k++) wmax = fmaxf(a.pred[k * n + i], wmax);
        double wsum = 0.0;
        float e[KR > 0 ? KR : 1];
        if (KR > 0) {
#pragma unroll
            for (int k = 0; k < KR; k++) {
                if ((uint32_t)k < K) {
                    e[k] = ex(__fsub_rn(a.pred[k * n + i], wmax));
                    wsum = __dadd_rn(wsum, (double)e[k]);
                }
            }
        } else {
            for (uint32_t k = 0; k < K; k++) wsum = __dadd_rn(wsum, (double)ex(__fsub_rn(a.pred[k * n + i], wmax)));
        }
        const float d = __double2float_rn(wsum);
        const float label = a.label[i];
        const float wt = a.weight ? a.weight[i] : 1.0f;
        auto emit = [&](uint32_t k, float ek) {
            float p = __fdiv_rn(ek, d);
            const float h = fmaxf(__fmul_rn(__fmul_rn(__fmul_rn(2.0f, p), __fsub_rn(1.0f, p)), wt), 1e-16f);
            if (label == (float)k) p = __fsub_rn(p, 1.0f);
            out[2 * (k * n + i)] = __fmul_rn(p, wt);
            out[2 * (k * n + i) + 1] = h;
        };
        if (KR > 0) {
#pragma unroll
            for (int k = 0; k < KR; k++)
                if ((uint32_t)k < K) emit((uint32_t)k, e[k]);
        } else {
            for (uint32_t k = 0; k < K; k++) emit(k, ex(__fsub_rn(a.pred[k * n + i], wmax)));
        }
    }
}

// Zero scales (a non-finite bound, k_device_scales_exact) quantize every
// row to zero.
__global__ void k_quantize(GradArgs a) {
    Pair s{0, 0};
    double gs = a.scales[0], hs = a.scales[1];
    const bool zero = gs == 0.0 || hs == 0.0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += blockDim.x * gridDim.x) {
        Pair f = zero ? Pair{0, 0} : to_fixed(a.gpair_f32[2ull * i], a.gpair_f32[2ull * i + 1], gs, hs);
        a.fixed[i] = f;
        s = padd(s, f);
    }
    fold_sum(s, a.sum);
}

// Fast mode: power-of-two scale on the device.  floor(log2(raw)) is taken as
// the binary exponent (ilogb), as the reference device path does
// (backend/cuda/histogram.cu:1179-1202); fast mode makes no byte-identity claim.
__device__ double d_pow2_scale(double max_abs, unsigned long long n_rows) {
    if (!(max_abs > 0.0) || !isfinite(max_abs)) return 1.0;
    double budget = __ddiv_rn(4611686018427387904.0, (double)(n_rows > 0 ? n_rows : 1));
    double raw = __ddiv_rn(budget, max_abs);
    if (!isfinite(raw) || raw <= 0.0) return 1.0;
    int k = ilogb(raw);
    k = k < -1000 ? -1000 : (k > 1000 ? 1000 : k);
    return ldexp(1.0, k);
}
// A non-finite bound: zero scales and *err = 1, as k_device_scales_exact.
__global__ void k_device_scales(const unsigned long long* maxbits, unsigned long long n_rows, double* scales,
                                unsigned long long* err) {
    const double mg = __longlong_as_double((long long)maxbits[0]), mh = __longlong_as_double((long long)maxbits[1]);
    if (!isfinite(mg) || !isfinite(mh)) {
        scales[0] = 0.0;
        scales[1] = 0.0;
        *err = 1ull;
        return;
    }
    scales[0] = d_pow2_scale(mg, n_rows);
    scales[1] = d_pow2_scale(mh, n_rows);
    *err = 0ull;
}

// Exact mode: the reference's scales (types.rs:366-385, the host's log2;
// qscale.h) from the bounds, so the round needs no host round trip.  A
// non-finite bound sets *err and zero scales: every fixed-point gradient is
// then zero (k_quantize), the tree grown from them adds nothing to the
// margins, and the host raises the error when it reads the tree back.
__global__ void k_device_scales_exact(const unsigned long long* maxbits, unsigned long long n_rows,
                                      const fbx::ScaleExc* exc, uint32_t n_exc, double* scales,
                                      unsigned long long* err) {
    const double mg = __longlong_as_double((long long)maxbits[0]), mh = __longlong_as_double((long long)maxbits[1]);
    if (!isfinite(mg) || !isfinite(mh)) {
        scales[0] = 0.0;
        scales[1] = 0.0;
        *err = 1ull;
        return;
    }
    scales[0] = fbx::scale_of_exp(fbx::scale_exp_exact(mg, n_rows, exc, n_exc));
    scales[1] = fbx::scale_of_exp(fbx::scale_exp_exact(mh, n_rows, exc, n_exc));
    *err = 0ull;
}

// The same scale of each value (the exactness tests).
__global__ void k_quantizer_scales(const float* vals, uint64_t count, unsigned long long n_rows,
                                   const fbx::ScaleExc* exc, uint32_t n_exc, double* out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)blockDim.x * gridDim.x)
        out[i] = fbx::scale_of_exp(fbx::scale_exp_exact((double)vals[i], n_rows, exc, n_exc));
}

// ------------------------------------------------------------------ histogram
// Exact i64 histograms in shared memory as four 32-bit planes (g_lo, g_hi,
// h_lo, h_hi).  A 64-bit add is a low-word atomic whose returned old value
// gives the carry, then a high-word atomic of (hi + carry); the planes then
// hold exactly the modulo-2^64 sums (hist.rs:94-274 semantics), whatever the
// order of the additions.
__device__ __forceinline__ void plane_add(uint32_t* lo, uint32_t* hi, uint32_t idx, long long v) {
    uint32_t vl = (uint32_t)v;
    uint32_t vh = (uint32_t)((unsigned long long)v >> 32);
    uint32_t old = atomicAdd(&lo[idx], vl);
    vh += (uint32_t)(old + vl < old);
    if (vh) atomicAdd(&hi[idx], vh);
}

template <int W>
__global__ void __launch_bounds__(kHistThreads) k_hist(const TileDesc* __restrict__ tiles,
                                                       const TileFeat* __restrict__ tfeat,
                                                       const uint32_t* __restrict__ rows,
                                                       const Pair* __restrict__ gpair,
                                                       const NodeInfo* __restrict__ nodes,
                                                       const uint32_t* __restrict__ acc_list,
                                                       const unsigned long long* __restrict__ acc_prefix,
                                                       const TreeState* __restrict__ st, Pair* __restrict__ hist_acc,
                                                       unsigned long long slot_pairs) {
    extern __shared__ uint32_t sm[];
    const TileDesc td = tiles[blockIdx.y];
    const uint32_t LB = td.local_bins;
    uint32_t* glo = sm;
    uint32_t* ghi = sm + LB;
    uint32_t* hlo = sm + 2 * LB;
    uint32_t* hhi = sm + 3 * LB;
    TileFeat* tf = reinterpret_cast<TileFeat*>(sm + 4 * LB);
    const unsigned long long R = st->acc_total;
    const uint32_t n_acc = st->acc_count;
    if (R == 0) return;
    unsigned long long a = R * blockIdx.x / gridDim.x;
    const unsigned long long b = R * (blockIdx.x + 1) / gridDim.x;
    if (a >= b) return;
    for (uint32_t t = threadIdx.x; t < td.n_feat; t += blockDim.x) tf[t] = tfeat[td.feat_begin + t];
    for (uint32_t j = threadIdx.x; j < 4 * LB; j += blockDim.x) sm[j] = 0u;
    __syncthreads();
    const uint32_t nf = td.n_feat;
    // a tile with no shared histogram (features wider than the shared-memory
    // budget, e.g. categorical features of tens of thousands of codes) adds
    // every update straight to the node histogram: 64-bit global atomics,
    // exact modulo 2^64 like the shared planes
    const bool direct = LB == 0;
    uint32_t k = find_segment(acc_prefix, n_acc, a);
    while (a < b) {
        const uint32_t node = acc_list[k];
        const NodeInfo ni = nodes[node];
        const unsigned long long seg_end = min(b, acc_prefix[k + 1]);
        const uint32_t base = ni.start + (uint32_t)(a - acc_prefix[k]);
        const uint32_t cnt = (uint32_t)(seg_end - a);
        const unsigned long long rs = st->rank_stride;
        for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
            const uint32_t r = rows[base + i];
            const Pair gp = gpair[r];
            const uint8_t* rec = td.base + (size_t)r * td.stride;
            for (uint32_t t = 0; t < nf; t++) {
                const TileFeat f = tf[t];
                uint32_t bin = W == 2 ? (uint32_t)(*reinterpret_cast<const uint16_t*>(rec + f.byte_off))
                                      : (uint32_t)rec[f.byte_off];
                if (bin >= f.nbins) continue;  // missing sentinels lie at or above every feature's bin count
                if (direct) {
                    Pair* o = acc_bin(hist_acc, ni.acc_slot, slot_pairs, rs, f.global_off + bin);
                    atomicAdd(reinterpret_cast<unsigned long long*>(&o->g), (unsigned long long)gp.g);
                    atomicAdd(reinterpret_cast<unsigned long long*>(&o->h), (unsigned long long)gp.h);
                    continue;
                }
                const uint32_t idx = f.local_off + bin;
                plane_add(glo, ghi, idx, gp.g);
                plane_add(hlo, hhi, idx, gp.h);
            }
        }
        if (direct) {
            a = seg_end;
            k++;
            continue;
        }
        __syncthreads();
        // flush: one 64-bit global atomic per non-zero word, then clear
        for (uint32_t j = threadIdx.x; j < LB; j += blockDim.x) {
            unsigned long long g = ((unsigned long long)ghi[j] << 32) | glo[j];
            unsigned long long h = ((unsigned long long)hhi[j] << 32) | hlo[j];
            if (g | h) {
                uint32_t lo = 0, hi = nf;
                while (hi - lo > 1) {
                    uint32_t mid = (lo + hi) >> 1;
                    if (tf[mid].local_off <= j) lo = mid; else hi = mid;
                }
                Pair* o = acc_bin(hist_acc, ni.acc_slot, slot_pairs, rs, tf[lo].global_off + (j - tf[lo].local_off));
                if (g) atomicAdd(reinterpret_cast<unsigned long long*>(&o->g), g);
                if (h) atomicAdd(reinterpret_cast<unsigned long long*>(&o->h), h);
                glo[j] = 0u; ghi[j] = 0u; hlo[j] = 0u; hhi[j] = 0u;
            }
        }
        __syncthreads();
        a = seg_end;
        k++;
    }
}

// Lane-per-feature histogram.  A warp takes kLpfRows consecutive arena rows at
// a time; lane t owns tile feature t (at most 32 per tile), so one row's bins
// arrive with a single coalesced record load.  The shared histogram is laid
// out [bin][32 lanes] per plane, so the 32 lanes of an atomic instruction
// always fall in 32 distinct banks: no bank conflicts whatever the bins.
constexpr int kLpfRows = 8;

template <int W>
__global__ void __launch_bounds__(kHistLpfThreads) k_hist_lpf(const TileDesc* __restrict__ tiles,
                                                               const TileFeat* __restrict__ tfeat,
                                                               const uint32_t* __restrict__ rows,
                                                               const Pair* __restrict__ gpair,
                                                               const NodeInfo* __restrict__ nodes,
                                                               const uint32_t* __restrict__ acc_list,
                                                               const unsigned long long* __restrict__ acc_prefix,
                                                               const TreeState* __restrict__ st,
                                                               Pair* __restrict__ hist_acc,
                                                               unsigned long long slot_pairs) {
    extern __shared__ uint32_t sm[];
    const TileDesc td = tiles[blockIdx.y];
    const uint32_t LB = td.local_bins;  // max bins of the tile x 32
    uint32_t* glo = sm;
    uint32_t* ghi = sm + LB;
    uint32_t* hlo = sm + 2 * LB;
    uint32_t* hhi = sm + 3 * LB;
    const unsigned long long R = st->acc_total;
    const uint32_t n_acc = st->acc_count;
    if (R == 0) return;
    unsigned long long a = R * blockIdx.x / gridDim.x;
    const unsigned long long b = R * (blockIdx.x + 1) / gridDim.x;
    if (a >= b) return;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const uint32_t nf = td.n_feat;
    TileFeat f{0, 0, 0, 0};
    if (lane < nf) f = tfeat[td.feat_begin + lane];
    const bool active = lane < nf;
    for (uint32_t j = threadIdx.x; j < 4 * LB; j += blockDim.x) sm[j] = 0u;
    __syncthreads();
    uint32_t k = find_segment(acc_prefix, n_acc, a);
    while (a < b) {
        const uint32_t node = acc_list[k];
        const NodeInfo ni = nodes[node];
        const unsigned long long seg_end = min(b, acc_prefix[k + 1]);
        const uint32_t* seg_rows = rows + ni.start + (uint32_t)(a - acc_prefix[k]);
        const uint32_t cnt = (uint32_t)(seg_end - a);
        for (uint32_t base = warp * kLpfRows; base < cnt; base += nwarps * kLpfRows) {
            const uint32_t kk = min((uint32_t)kLpfRows, cnt - base);
            const uint32_t rid = lane < kk ? seg_rows[base + lane] : 0u;
            uint32_t bin[kLpfRows];
            Pair gp[kLpfRows];
#pragma unroll
            for (int q = 0; q < kLpfRows; q++) {
                const uint32_t r = __shfl_sync(0xffffffffu, rid, q);
                bin[q] = 0xffffffffu;
                gp[q] = Pair{0, 0};
                if ((uint32_t)q < kk) {
                    gp[q] = gpair[r];
                    if (active) {
                        const uint8_t* p = td.base + (size_t)r * td.stride + f.byte_off;
                        bin[q] = W == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < kLpfRows; q++) {
                if (bin[q] < f.nbins) {  // missing sentinels lie at or above every feature's bin count
                    const uint32_t idx = bin[q] * 32u + lane;
                    plane_add(glo, ghi, idx, gp[q].g);
                    plane_add(hlo, hhi, idx, gp[q].h);
                }
            }
        }
        __syncthreads();
        const unsigned long long rs = st->rank_stride;
        for (uint32_t j = threadIdx.x; j < LB; j += blockDim.x) {
            const unsigned long long g = ((unsigned long long)ghi[j] << 32) | glo[j];
            const unsigned long long h = ((unsigned long long)hhi[j] << 32) | hlo[j];
            if (g | h) {
                const uint32_t t = j & 31u, bb = j >> 5;
                const TileFeat ft = tfeat[td.feat_begin + t];
                Pair* o = acc_bin(hist_acc, ni.acc_slot, slot_pairs, rs, ft.global_off + bb);
                if (g) atomicAdd(reinterpret_cast<unsigned long long*>(&o->g), g);
                if (h) atomicAdd(reinterpret_cast<unsigned long long*>(&o->h), h);
                glo[j] = 0u; ghi[j] = 0u; hlo[j] = 0u; hhi[j] = 0u;
            }
        }
        __syncthreads();
        a = seg_end;
        k++;
    }
}

// Staged lane-per-feature histogram.  As in k_hist_lpf, lane t of a warp
// owns tile feature t and the shared histogram is laid out [bin][32 lanes].
// The difference is how rows reach the lanes: each warp keeps S batches of
// kStageRows rows in flight through cp.async (16-byte copies into shared
// memory, cached in L2 only): for every row the 16-byte chunks of its record
// that hold the tile's bins, and its 16-byte gradient pair.  A batch is
// consumed from shared memory while the next S-1 are still arriving, so a
// warp never stalls on one row's gather, and no registers hold loads in
// flight.  Row ids come in coalesced 32-row loads, one super-batch (4
// batches) ahead.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// 64-bit modular add into a (low, high) pair of 32-bit shared words: the low
// atomic returns the old word, whose sum with the addend's low word gives the
// carry; the high atomic always runs, so no branch depends on the value.
__device__ __forceinline__ void add64_planes(uint32_t* lo, uint32_t* hi, long long v) {
    const uint32_t vl = (uint32_t)v, vh = (uint32_t)((unsigned long long)v >> 32);
    const uint32_t old = atomicAdd(lo, vl);
    uint32_t sum, hi_add;
    asm("add.cc.u32 %0, %2, %3;\n\taddc.u32 %1, %4, 0;" : "=r"(sum), "=r"(hi_add) : "r"(old), "r"(vl), "r"(vh));
    (void)sum;
    atomicAdd(hi, hi_add);
}

// The high-word addend of a 64-bit add whose low word went through a
// returning atomic that found `old`: the addend's high word plus the carry.
__device__ __forceinline__ uint32_t carry_into_high(uint32_t old, long long v) {
    const uint32_t vl = (uint32_t)v, vh = (uint32_t)((unsigned long long)v >> 32);
    uint32_t sum, hi_add;
    asm("add.cc.u32 %0, %2, %3;\n\taddc.u32 %1, %4, 0;" : "=r"(sum), "=r"(hi_add) : "r"(old), "r"(vl), "r"(vh));
    (void)sum;
    return hi_add;
}
constexpr uint32_t kHistGroup = 4;

template <int W, int S, int LPR>
__global__ void __launch_bounds__(kHistLpfThreads) k_hist_stage(const TileDesc* __restrict__ tiles,
                                                                 const TileFeat* __restrict__ tfeat,
                                                                 const uint32_t* __restrict__ rows,
                                                                 const Pair* __restrict__ gpair,
                                                                 const NodeInfo* __restrict__ nodes,
                                                                 const uint32_t* __restrict__ acc_list,
                                                                 const unsigned long long* __restrict__ acc_prefix,
                                                                 const TreeState* __restrict__ st,
                                                                 Pair* __restrict__ hist_acc,
                                                                 unsigned long long slot_pairs) {
    extern __shared__ __align__(16) uint32_t sm[];
    const TileDesc td = tiles[blockIdx.y];
    const uint32_t LB = td.local_bins;  // max bins of the tile x LPR
    // LPR = 32 (features up to 440 bins): lane t of a warp owns tile feature
    // t; words laid out [bin][plane g_lo, g_hi, h_lo, h_hi][32 lanes], so one
    // address per (bin, lane) reaches all four planes by fixed offsets and the
    // 32 lanes of an atomic fall in 32 distinct banks.
    // LPR = 8 (wide features, up to 1024 bins): a warp takes 4 rows at a time,
    // lanes 8g..8g+7 the 8 tile features of row g; words laid out
    // [plane][bin][8 lanes] (bins padded to a multiple of 4), so a lane's bank
    // is 8 (bin mod 4) + feature and the four rows spread over the banks by
    // their bins.
    const unsigned long long R = st->acc_total;
    const uint32_t n_acc = st->acc_count;
    if (R == 0) return;
    unsigned long long a = R * blockIdx.x / gridDim.x;
    const unsigned long long b = R * (blockIdx.x + 1) / gridDim.x;
    if (a >= b) return;
    constexpr uint32_t G = 32 / LPR;  // rows per step
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const uint32_t tl = lane % LPR, grp = lane / LPR;
    const uint32_t nf = td.n_feat, nch = td.n_chunks;
    const uint32_t MB = LB / LPR;                       // bins per feature slot (discard row = MB)
    const uint32_t PS = ((MB + 1 + 3) & ~3u) * LPR;     // words per plane (LPR = 8)
    const uint32_t hist_words = LPR == 32 ? 4 * (LB + 32) : 4 * PS;
    uint32_t* hlane = sm + tl;
    const uint32_t rec_bytes = nch * 16u;
    const uint32_t stage_bytes = kStageRows * (rec_bytes + 16u);
    // bins 0 .. MB - 1, then one discard row that missing bins and idle
    // lanes add to, so the row loop has no branch on the bin
    const uint32_t discard = MB;
    uint8_t* wbuf = reinterpret_cast<uint8_t*>(sm + hist_words) + (size_t)warp * S * stage_bytes;
    TileFeat f{0, 0, 0, 0};
    if (tl < nf) f = tfeat[td.feat_begin + tl];
    const bool active = tl < nf;
    const uint32_t foff = active ? f.byte_off - td.chunk0 * 16u : 0u;
    // the missing sentinel (255 / 65535) is never below a feature's bin count
    const uint32_t nbins = active ? f.nbins : 0u;
    const uint8_t* rec_base = td.base + td.chunk0 * 16u;
    // copy assignment: lane = (item group g, row q); items of a row are its
    // record chunks 0..nch-1 and its gradient pair (item nch)
    const uint32_t cq = lane & 7u, cg = lane >> 3;
    for (uint32_t j = threadIdx.x; j < (LPR == 32 ? 4 * LB : hist_words); j += blockDim.x) sm[j] = 0u;
    __syncthreads();
    uint32_t k = find_segment(acc_prefix, n_acc, a);
    while (a < b) {
        const uint32_t node = acc_list[k];
        const NodeInfo ni = nodes[node];
        const unsigned long long seg_end = min(b, acc_prefix[k + 1]);
        const uint32_t* seg_rows = rows + ni.start + (uint32_t)(a - acc_prefix[k]);
        const uint32_t cnt = (uint32_t)(seg_end - a);
        // this warp's super-batches: 32 rows each, sb = warp, warp + nwarps, ...
        const uint32_t n_sb = (cnt + 31) / 32;
        const uint32_t my_sb = warp < n_sb ? (n_sb - warp + nwarps - 1) / nwarps : 0u;
        const uint32_t nb = my_sb * 4;
        auto load_ids = [&](uint32_t kk) -> uint32_t {
            const uint32_t r = (warp + kk * nwarps) * 32u + lane;
            return (kk < my_sb && r < cnt) ? seg_rows[r] : 0u;
        };
        uint32_t ids_cur = load_ids(0), ids_nxt = load_ids(1), k_cur = 0;
        auto issue = [&](uint32_t bb) {
            if (bb < nb) {
                const uint32_t kk = bb >> 2, sub = bb & 3u;
                const uint32_t ids = kk == k_cur ? ids_cur : ids_nxt;
                const uint32_t first = (warp + kk * nwarps) * 32u + sub * kStageRows;
                const uint32_t kq = first < cnt ? min(kStageRows, cnt - first) : 0u;
                const uint32_t rid = __shfl_sync(0xffffffffu, ids, sub * kStageRows + cq);
                uint8_t* stg = wbuf + (bb % S) * stage_bytes;
                if (cq < kq) {
                    for (uint32_t it = cg; it <= nch; it += 4) {
                        if (it < nch)
                            cp_async16(stg + cq * rec_bytes + it * 16u, rec_base + (size_t)rid * td.stride + it * 16u);
                        else
                            cp_async16(stg + kStageRows * rec_bytes + cq * 16u, gpair + rid);
                    }
                }
            }
            cp_async_commit();
        };
#pragma unroll
        for (int s0 = 0; s0 < S; s0++) issue((uint32_t)s0);
        for (uint32_t bb = 0; bb < nb; bb++) {
            if (bb > 0 && (bb & 3u) == 0) {  // next super-batch: rotate the prefetched ids
                k_cur++;
                ids_cur = ids_nxt;
                ids_nxt = load_ids(k_cur + 1);
            }
            cp_async_wait<S - 1>();
            __syncwarp();
            const uint32_t first = (warp + (bb >> 2) * nwarps) * 32u + (bb & 3u) * kStageRows;
            const uint32_t kq = first < cnt ? min(kStageRows, cnt - first) : 0u;
            const uint8_t* stg = wbuf + (bb % S) * stage_bytes;
            const Pair* gps = reinterpret_cast<const Pair*>(stg + kStageRows * rec_bytes);
            const uint8_t* pr = stg + foff;
            auto row = [&](uint32_t q) {
                const uint8_t* p = pr + q * rec_bytes;
                uint32_t bin = W == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
                bin = bin < nbins ? bin : discard;
                const Pair gp = gps[q];
                if (LPR == 32) {
                    uint32_t* w = hlane + bin * 128u;
                    add64_planes(w, w + 32, gp.g);
                    add64_planes(w + 64, w + 96, gp.h);
                } else {
                    uint32_t* w = hlane + bin * LPR;
                    add64_planes(w, w + PS, gp.g);
                    add64_planes(w + 2 * PS, w + 3 * PS, gp.h);
                }
            };
            if (LPR == 32) {
                if (kq == kStageRows) {
                    // kHistGroup rows at a time: their returning low-word atomics
                    // first, then the high words with the carries, so several
                    // returns are in flight instead of one chain per row (the
                    // carries are per atomic, so any interleaving sums exactly)
#pragma unroll
                    for (uint32_t q0 = 0; q0 < kStageRows; q0 += kHistGroup) {
                        uint32_t* wq[kHistGroup];
                        Pair gq[kHistGroup];
                        uint32_t og[kHistGroup], oh[kHistGroup];
#pragma unroll
                        for (uint32_t u = 0; u < kHistGroup; u++) {
                            const uint8_t* p = pr + (q0 + u) * rec_bytes;
                            uint32_t bin = W == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
                            bin = bin < nbins ? bin : discard;
                            wq[u] = hlane + bin * 128u;
                            gq[u] = gps[q0 + u];
                        }
#pragma unroll
                        for (uint32_t u = 0; u < kHistGroup; u++) {
                            og[u] = atomicAdd(wq[u], (uint32_t)gq[u].g);
                            oh[u] = atomicAdd(wq[u] + 64, (uint32_t)gq[u].h);
                        }
#pragma unroll
                        for (uint32_t u = 0; u < kHistGroup; u++) {
                            atomicAdd(wq[u] + 32, carry_into_high(og[u], gq[u].g));
                            atomicAdd(wq[u] + 96, carry_into_high(oh[u], gq[u].h));
                        }
                    }
                } else {
                    for (uint32_t q = 0; q < kq; q++) row(q);
                }
            } else {
#pragma unroll
                for (uint32_t s2 = 0; s2 < kStageRows / G; s2++) {
                    const uint32_t q = s2 * G + grp;
                    if (q < kq) row(q);
                }
            }
            __syncwarp();
            issue(bb + S);
        }
        cp_async_wait<0>();
        __syncthreads();
        const unsigned long long rs = st->rank_stride;
        for (uint32_t j = threadIdx.x; j < LB; j += blockDim.x) {
            const uint32_t t = j % LPR, bb = j / LPR;
            uint32_t* w = LPR == 32 ? sm + bb * 128u + t : sm + bb * LPR + t;
            const uint32_t o1 = LPR == 32 ? 32u : PS, o2 = LPR == 32 ? 64u : 2 * PS, o3 = LPR == 32 ? 96u : 3 * PS;
            const unsigned long long g = ((unsigned long long)w[o1] << 32) | w[0];
            const unsigned long long h = ((unsigned long long)w[o3] << 32) | w[o2];
            if (g | h) {
                const TileFeat ft = tfeat[td.feat_begin + t];
                Pair* o = acc_bin(hist_acc, ni.acc_slot, slot_pairs, rs, ft.global_off + bb);
                if (g) atomicAdd(reinterpret_cast<unsigned long long*>(&o->g), g);
                if (h) atomicAdd(reinterpret_cast<unsigned long long*>(&o->h), h);
                w[0] = 0u; w[o1] = 0u; w[o2] = 0u; w[o3] = 0u;
            }
        }
        __syncthreads();
        a = seg_end;
        k++;
    }
}

// ------------------------------------------------------------------ split
// Wide categorical features (more codes than the split CTA has threads, up to
// 65534 codes: categorical.rs:19-28 MAX_CAT_CODE_WIDE).  The reference sorts
// all codes stably by weight and scans the first and the last n_scan - 1 of
// that order (split.rs:484-617).  Only those codes take part, so instead of
// sorting every code the CTA selects them by rank: a code's order key is its
// f32 weight mapped to an order-preserving u32 (-0 and +0 one key, as `<`
// sees them) with the code as the tie break; the key of a given rank comes
// from a 4-pass radix select over the weight keys and a search in code order
// among equal weights; each tile of kCatTile ranks is gathered into shared
// memory, sorted, and scanned with the carry of the tiles before it.
constexpr uint32_t kCatTile = 512;

struct CatWideSmem {
    unsigned long long key[kCatTile];  // a tile's composite keys (weight key << 32 | code)
    uint32_t digit[256];
    uint32_t count, sel_digit, sel_before, sel_code;
};

struct SplitSmem {
    Pair warp_tot[32];
    SplitRec best[kSplitThreads];
    union {
        struct {
            float w[kSplitThreads];
            uint32_t idx[kSplitThreads];
            Pair x[kSplitThreads];  // the finished histogram (parent and child may share memory)
        } c;                        // categorical features of at most kSplitThreads codes
        CatWideSmem wide;           // wider categorical features
    } u;
    uint32_t set_words[8];
    uint32_t wt[32];
};

__device__ __forceinline__ void consider(SplitRec& best, float gain, uint32_t ord, uint32_t bin, uint32_t flags,
                                         Pair l, Pair r) {
    if (!(gain > 1e-6f)) return;  // split.rs:260-270 update_best (NaN filtered too)
    if (!(best.flags & 1u) || gain > best.gain || (gain == best.gain && ord < best.ord)) {
        best.gain = gain; best.ord = ord; best.bin = bin; best.flags = flags | 1u;
        best.left = l; best.right = r;
    }
}

__device__ __forceinline__ void block_best(SplitSmem& s, SplitRec& mine) {
    s.best[threadIdx.x] = mine;
    __syncthreads();
    for (int stride = kSplitThreads / 2; stride > 0; stride >>= 1) {
        if ((int)threadIdx.x < stride && rec_better(s.best[threadIdx.x + stride], s.best[threadIdx.x]))
            s.best[threadIdx.x] = s.best[threadIdx.x + stride];
        __syncthreads();
    }
}

// A category's sort key: its weight (CalcWeightCat, split.rs:520-530) as an
// order-preserving u32.
__device__ __forceinline__ uint32_t cat_weight_key(Pair x, const ScoreParams& sp) {
    float w = xgb_weight(to_f64(x.g, sp.inv_g), to_f64(x.h, sp.inv_h), sp);
    if (w == 0.0f) w = 0.0f;  // -0 and +0 compare equal under the sort's `<`: one key
    const uint32_t b = __float_as_uint(w);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ unsigned long long cat_order_key(const Pair* hx, uint32_t c, const ScoreParams& sp) {
    return ((unsigned long long)cat_weight_key(hx[c], sp) << 32) | c;
}

// The order key of the code with exactly r codes before it in the stable
// weight order (0 <= r < n).  Every thread of the CTA calls it.
__device__ unsigned long long cat_select(const Pair* hx, uint32_t n, const ScoreParams& sp, uint32_t r,
                                         SplitSmem& s) {
    CatWideSmem& ws = s.u.wide;
    uint32_t prefix = 0, mask = 0, rem = r;
    for (int shift = 24; shift >= 0; shift -= 8) {
        ws.digit[threadIdx.x] = 0u;  // blockDim == 256 == digits
        __syncthreads();
        for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) {
            const uint32_t k = cat_weight_key(hx[c], sp);
            if ((k & mask) == prefix) atomicAdd(&ws.digit[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        const uint32_t cnt = ws.digit[threadIdx.x];
        uint32_t tot;
        const uint32_t before = block_excl_scan_u32<kSplitThreads>(cnt, s.wt, tot);
        if (before <= rem && rem < before + cnt) {
            ws.sel_digit = threadIdx.x;
            ws.sel_before = before;
        }
        __syncthreads();
        rem -= ws.sel_before;
        prefix |= ws.sel_digit << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    // the rem-th code, in code order, among those whose weight key is `prefix`
    uint32_t seen = 0;
    for (uint32_t base = 0; base < n; base += blockDim.x) {
        const uint32_t c = base + threadIdx.x;
        const bool match = c < n && cat_weight_key(hx[c], sp) == prefix;
        uint32_t tot;
        const uint32_t ex = block_excl_scan_u32<kSplitThreads>(match ? 1u : 0u, s.wt, tot);
        if (match && seen + ex == rem) ws.sel_code = c;
        seen += tot;
        if (seen > rem) break;  // uniform: every thread holds the same `seen`
    }
    __syncthreads();
    const uint32_t code = ws.sel_code;
    __syncthreads();
    return ((unsigned long long)prefix << 32) | code;
}

// Gathers the codes whose order keys lie in [lo, hi) (at most kCatTile) into
// ws.key, sorted ascending; returns how many.
__device__ uint32_t cat_gather(const Pair* hx, uint32_t n, const ScoreParams& sp, unsigned long long lo,
                               unsigned long long hi, SplitSmem& s) {
    CatWideSmem& ws = s.u.wide;
    if (threadIdx.x == 0) ws.count = 0u;
    __syncthreads();
    for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) {
        const unsigned long long k = cat_order_key(hx, c, sp);
        if (k >= lo && k < hi) {
            const uint32_t at = atomicAdd(&ws.count, 1u);
            if (at < kCatTile) ws.key[at] = k;
        }
    }
    __syncthreads();
    const uint32_t cnt = min(ws.count, kCatTile);
    for (uint32_t i = cnt + threadIdx.x; i < kCatTile; i += blockDim.x) ws.key[i] = ~0ull;
    __syncthreads();
    for (uint32_t size = 2; size <= kCatTile; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = threadIdx.x; i < kCatTile; i += blockDim.x) {
                const uint32_t j = i ^ stride;
                if (j > i) {
                    const unsigned long long x = ws.key[i], y = ws.key[j];
                    if ((x > y) == ((i & size) == 0)) { ws.key[i] = y; ws.key[j] = x; }
                }
            }
            __syncthreads();
        }
    }
    return cnt;
}

// Best categorical split of a feature with n > kSplitThreads codes whose
// finished histogram is hx[0..n) (split.rs:484-617: one-hot below
// max_cat_to_onehot, else the partition scans), and its right-going set
// written to cw (cat_words words).
__device__ void split_cat_wide(const LevelArgs& a, SplitSmem& s, const Pair* hx, uint32_t n, Pair sum,
                               float parent_gain, int cons, const NodeInfo& ni, const ScoreParams& sp, SplitRec& mine,
                               uint32_t* cw) {
    const uint32_t W = a.cat_words;
    if (n < a.max_onehot) {
        Pair loc{0, 0};
        for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) loc = padd(loc, hx[c]);
        Pair tot;
        (void)block_excl_scan_pair<kSplitThreads>(loc, s.warp_tot, tot);
        const Pair missing = psub(sum, tot);
        for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) {
            const Pair x = hx[c];
            float gain;
            Pair l = psub(sum, x);
            if (split_gain(parent_gain, l, x, cons, ni.lower, ni.upper, sp, gain))
                consider(mine, gain, 2 * c, c, 2u | 4u, l, x);
            const Pair r = padd(x, missing);
            l = psub(sum, r);
            if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                consider(mine, gain, 2 * c + 1, c, 4u, l, r);
        }
        block_best(s, mine);
        const SplitRec b = s.best[0];
        for (uint32_t w = threadIdx.x; w < W; w += blockDim.x)
            cw[w] = (b.flags & 1u) && w == (b.bin >> 5) ? 1u << (b.bin & 31) : 0u;
        return;
    }
    const uint32_t n_scan = min(a.max_cat_threshold, n);
    const uint32_t K = n_scan >= 2 ? n_scan - 1 : 0u;
    // forward: the first t+1 codes of the order go right, missing left
    Pair carry{0, 0};
    unsigned long long t_lo = 0ull;
    for (uint32_t lo = 0; lo < K; lo += kCatTile) {
        const uint32_t hi = min(lo + kCatTile, K);
        const unsigned long long t_hi = cat_select(hx, n, sp, hi, s);
        const uint32_t cnt = cat_gather(hx, n, sp, t_lo, t_hi, s);
        const uint32_t i0 = 2 * threadIdx.x;
        const Pair x0 = i0 < cnt ? hx[(uint32_t)s.u.wide.key[i0]] : Pair{0, 0};
        const Pair x1 = i0 + 1 < cnt ? hx[(uint32_t)s.u.wide.key[i0 + 1]] : Pair{0, 0};
        Pair tot;
        const Pair ex = block_excl_scan_pair<kSplitThreads>(padd(x0, x1), s.warp_tot, tot);
        Pair run = padd(carry, ex);
        for (uint32_t q = 0; q < 2; q++) {
            const uint32_t i = i0 + q;
            run = padd(run, q ? x1 : x0);
            if (i < cnt) {
                const uint32_t rank = lo + i;
                const Pair r = run, l = psub(sum, r);
                float gain;
                if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, rank, rank + 1, 2u | 4u, l, r);
            }
        }
        carry = padd(carry, tot);
        t_lo = t_hi;
        __syncthreads();
    }
    // backward: the order's tail from rank t goes left, missing right
    carry = Pair{0, 0};
    unsigned long long t_hi = ~0ull;
    for (uint32_t hi = n; K && hi > n - K;) {
        const uint32_t lo = max(n - K, hi > kCatTile ? hi - kCatTile : 0u);
        const unsigned long long t_lo2 = cat_select(hx, n, sp, lo, s);
        const uint32_t cnt = cat_gather(hx, n, sp, t_lo2, t_hi, s);
        const uint32_t i0 = 2 * threadIdx.x;
        const Pair x0 = i0 < cnt ? hx[(uint32_t)s.u.wide.key[i0]] : Pair{0, 0};
        const Pair x1 = i0 + 1 < cnt ? hx[(uint32_t)s.u.wide.key[i0 + 1]] : Pair{0, 0};
        Pair tot;
        const Pair ex = block_excl_scan_pair<kSplitThreads>(padd(x0, x1), s.warp_tot, tot);
        Pair before = ex;  // this tile's codes ranked before element i
        for (uint32_t q = 0; q < 2; q++) {
            const uint32_t i = i0 + q;
            if (i < cnt) {
                const uint32_t rank = lo + i;
                const Pair l = padd(carry, psub(tot, before)), r = psub(sum, l);
                float gain;
                if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, (n_scan - 1) + (n - 1 - rank), rank, 4u, l, r);
            }
            before = padd(before, q ? x1 : x0);
        }
        carry = padd(carry, tot);
        t_hi = t_lo2;
        hi = lo;
        __syncthreads();
    }
    block_best(s, mine);
    const SplitRec b = s.best[0];
    // the right-going set: the b.bin codes first in the order
    const unsigned long long cut = (b.flags & 1u) ? cat_select(hx, n, sp, b.bin, s) : 0ull;
    for (uint32_t w = threadIdx.x; w < W; w += blockDim.x) {
        uint32_t word = 0u;
        for (uint32_t k = 0; k < 32; k++) {
            const uint32_t c = 32 * w + k;
            if (c < n && cat_order_key(hx, c, sp) < cut) word |= 1u << k;
        }
        cw[w] = word;
    }
}

// Per (node, feature) CTA: finish the node histogram (copy or parent minus
// sibling), scan it, score every candidate and keep the first maximum in the
// reference's enumeration order (split.rs:331-461; categorical :484-617).
__global__ void __launch_bounds__(kSplitThreads) k_split_feat(LevelArgs a) {
    // features feat_lo.. (all features, unless the split search is feature-sharded);
    // with the warp kernel beside it, only the categorical and wide ones
    const uint32_t node = blockIdx.x, F = a.n_features;
    const uint32_t f = a.split_cta ? a.split_cta[blockIdx.y] : a.feat_lo + blockIdx.y;
    if (node >= a.st->m) return;
    SplitRec* out = a.feat_best + (size_t)node * F + f;
    if (!a.enabled[f] || f >= a.feat_hi) {
        if (threadIdx.x == 0) out->flags = 0;
        return;
    }
    __shared__ SplitSmem s;
    const NodeInfo ni = a.nodes[node];
    const uint32_t off = a.hoff[f] - a.bin_lo, nb = a.hoff[f + 1] - a.hoff[f];
    const Pair* acc = a.hist_acc + (unsigned long long)ni.acc_slot * a.slot_pairs + off;
    const Pair* par = ni.parent_slot >= 0 ? a.hist_prev + (unsigned long long)ni.parent_slot * a.slot_pairs + off
                                          : nullptr;
    // the subtracted child may be written over its parent's histogram (lossguide pool):
    // every bin is read once, by the thread that writes it
    Pair* h = a.hist_cur + (unsigned long long)(a.node_hist ? a.node_hist[node] : node) * a.slot_pairs + off;
    const bool keep_hist = !a.last_level;
    const Pair sum = ni.sum;
    const ScoreParams sp = load_sp(a);
    const float parent_gain = node_gain(sum, sp, ni.lower, ni.upper);
    const int cons = a.mono ? (int)a.mono[f] : 0;
    SplitRec mine;
    mine.flags = 0; mine.gain = 0.0f; mine.ord = 0xffffffffu; mine.bin = 0; mine.feat = f;
    mine.left = Pair{0, 0}; mine.right = Pair{0, 0};

    if (a.is_cat && a.is_cat[f]) {
        const uint32_t W = a.cat_words;
        uint32_t* cw = a.feat_cats + ((size_t)node * a.n_cat + a.cat_slot[f]) * W;
        if (nb > kSplitThreads) {
            // ---- wide categorical: the finished histogram goes to h first (each bin
            // read and written by one thread), then the rank-selected scans read it
            for (uint32_t c = threadIdx.x; c < nb; c += blockDim.x) h[c] = par ? psub(par[c], acc[c]) : acc[c];
            __syncthreads();
            split_cat_wide(a, s, h, nb, sum, parent_gain, cons, ni, sp, mine, cw);
            if (threadIdx.x == 0) {
                SplitRec b = s.best[0];
                b.feat = f;
                *out = b;
            }
            return;
        }
        // ---- categorical: one bin per category code, n <= 256 (one per thread)
        const uint32_t n = nb, t = threadIdx.x;
        Pair x{0, 0};
        if (t < n) {
            x = par ? psub(par[t], acc[t]) : acc[t];
            if (keep_hist) h[t] = x;
        }
        if (n < a.max_onehot) {
            Pair tot;
            (void)block_excl_scan_pair<kSplitThreads>(x, s.warp_tot, tot);
            const Pair missing = psub(sum, tot);
            if (t < n) {
                float gain;
                Pair l = psub(sum, x);
                if (split_gain(parent_gain, l, x, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, 2 * t, t, 2u | 4u, l, x);
                Pair r = padd(x, missing);
                l = psub(sum, r);
                if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, 2 * t + 1, t, 4u, l, r);
            }
            block_best(s, mine);
            const SplitRec b = s.best[0];
            for (uint32_t w = threadIdx.x; w < W; w += blockDim.x)
                cw[w] = (b.flags & 1u) && w == (b.bin >> 5) ? 1u << (b.bin & 31) : 0u;
            if (threadIdx.x == 0) {
                SplitRec bf = b;
                bf.feat = f;
                *out = bf;
            }
            return;
        }
        // partition mode: stable sort of categories by weight (CalcWeightCat)
        float w = __int_as_float(0x7f800000);
        if (t < n) w = xgb_weight(to_f64(x.g, sp.inv_g), to_f64(x.h, sp.inv_h), sp);
        s.u.c.w[t] = w;
        s.u.c.idx[t] = t;
        s.u.c.x[t] = x;
        __syncthreads();
        for (uint32_t size = 2; size <= kSplitThreads; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                uint32_t partner = t ^ stride;
                if (partner > t) {
                    bool up = (t & size) == 0;
                    float wa = s.u.c.w[t], wb = s.u.c.w[partner];
                    uint32_t ia = s.u.c.idx[t], ib = s.u.c.idx[partner];
                    // (weight, index) order == std::stable_sort by `<` on weight
                    bool a_gt_b = (wb < wa) || (!(wa < wb) && ib < ia);
                    if (a_gt_b == up) {
                        s.u.c.w[t] = wb; s.u.c.w[partner] = wa;
                        s.u.c.idx[t] = ib; s.u.c.idx[partner] = ia;
                    }
                }
                __syncthreads();
            }
        }
        const uint32_t cat = s.u.c.idx[t];
        Pair xs = t < n ? s.u.c.x[cat] : Pair{0, 0};
        Pair tot;
        Pair excl = block_excl_scan_pair<kSplitThreads>(xs, s.warp_tot, tot);
        const uint32_t n_scan = min(a.max_cat_threshold, n);
        if (n_scan >= 2 && t < n) {
            float gain;
            if (t + 1 < n_scan) {  // forward: first t+1 sorted categories go right, missing left
                Pair r = padd(excl, xs);
                Pair l = psub(sum, r);
                if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, t, t + 1, 2u | 4u, l, r);
            }
            if (t >= n - (n_scan - 1)) {  // backward: sorted tail from t goes left, missing right
                Pair l = psub(tot, excl);
                Pair r = psub(sum, l);
                if (split_gain(parent_gain, l, r, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, (n_scan - 1) + (n - 1 - t), t, 4u, l, r);
            }
        }
        block_best(s, mine);
        SplitRec b = s.best[0];
        if (t < 8) s.set_words[t] = 0u;
        __syncthreads();
        if ((b.flags & 1u) && t < b.bin) atomicOr(&s.set_words[cat >> 5], 1u << (cat & 31));
        __syncthreads();
        for (uint32_t wi = t; wi < W; wi += blockDim.x) cw[wi] = wi < 8 ? s.set_words[wi] : 0u;
        if (t == 0) {
            b.feat = f;
            *out = b;
        }
        return;
    }

    // ---- numeric feature: forward (missing right) then reverse (missing left)
    const uint32_t bpt = (nb + kSplitThreads - 1) / kSplitThreads;
    const uint32_t b0 = threadIdx.x * bpt;
    Pair v[kMaxBinsPerThread];
    Pair loc{0, 0};
#pragma unroll
    for (int k = 0; k < kMaxBinsPerThread; k++) {
        uint32_t bidx = b0 + k;
        Pair x{0, 0};
        if (k < (int)bpt && bidx < nb) {
            x = par ? psub(par[bidx], acc[bidx]) : acc[bidx];
            if (keep_hist) h[bidx] = x;
        }
        v[k] = x;
        loc = padd(loc, x);
    }
    Pair total;
    Pair run = block_excl_scan_pair<kSplitThreads>(loc, s.warp_tot, total);
    const bool reverse = !peq(total, sum);
#pragma unroll
    for (int k = 0; k < kMaxBinsPerThread; k++) {
        uint32_t bidx = b0 + k;
        if (k < (int)bpt && bidx < nb) {
            Pair excl = run;
            run = padd(run, v[k]);
            float gain;
            Pair r = psub(sum, run);
            if (split_gain(parent_gain, run, r, cons, ni.lower, ni.upper, sp, gain))
                consider(mine, gain, bidx, bidx + 1, 0u, run, r);
            if (reverse) {
                Pair rr = psub(total, excl);
                Pair ll = psub(sum, rr);
                if (split_gain(parent_gain, ll, rr, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, nb + (nb - 1 - bidx), bidx, 2u, ll, rr);
            }
        }
    }
    block_best(s, mine);
    if (threadIdx.x == 0) {
        SplitRec b = s.best[0];
        b.feat = f;
        *out = b;
    }
}

// Numeric features of at most kSplitWarpBins bins: one warp per (node,
// feature), lane l holding bins [8l, 8l + 8).  The same candidates as the
// numeric path of k_split_feat (forward with missing right at every bin,
// then, when the node has missing values, reverse with missing left; the
// same ordinals), the prefix sums and the arg-max by shuffles, so no block
// barrier.  The arg-max order (gain, then ordinal) is total, so the winner
// does not depend on how the candidates are reduced.
// 128-thread CTAs (16 resident warps per SM at the kernel's ~110 registers;
// bounding it further spills): a level's (node, feature) warps are spread
// in finer steps than with 256-thread CTAs.
constexpr uint32_t kSplitWarpBins = 256;
constexpr uint32_t kSplitNumThreads = 128;
__global__ void __launch_bounds__(kSplitNumThreads) k_split_num(LevelArgs a) {
    const uint32_t node = blockIdx.x, lane = threadIdx.x & 31u;
    const uint32_t item = blockIdx.y * (kSplitNumThreads / 32) + (threadIdx.x >> 5);
    if (node >= a.st->m || item >= a.n_split_num) return;
    const uint32_t f = a.split_num[item];
    SplitRec* out = a.feat_best + (size_t)node * a.n_features + f;
    if (!a.enabled[f]) {
        if (lane == 0) out->flags = 0;
        return;
    }
    const NodeInfo ni = a.nodes[node];
    const uint32_t off = a.hoff[f] - a.bin_lo, nb = a.hoff[f + 1] - a.hoff[f];
    const Pair* acc = a.hist_acc + (unsigned long long)ni.acc_slot * a.slot_pairs + off;
    const Pair* par = ni.parent_slot >= 0 ? a.hist_prev + (unsigned long long)ni.parent_slot * a.slot_pairs + off
                                          : nullptr;
    Pair* h = a.hist_cur + (unsigned long long)(a.node_hist ? a.node_hist[node] : node) * a.slot_pairs + off;
    const bool keep_hist = !a.last_level;
    const Pair sum = ni.sum;
    const ScoreParams sp = load_sp(a);
    const float parent_gain = node_gain(sum, sp, ni.lower, ni.upper);
    const int cons = a.mono ? (int)a.mono[f] : 0;
    const uint32_t b0 = lane * 8;
    Pair v[8];
    Pair loc{0, 0};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t bidx = b0 + k;
        Pair x{0, 0};
        if (bidx < nb) {
            x = par ? psub(par[bidx], acc[bidx]) : acc[bidx];
            if (keep_hist) h[bidx] = x;
        }
        v[k] = x;
        loc = padd(loc, x);
    }
    Pair incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const Pair t{__shfl_up_sync(0xffffffffu, incl.g, o), __shfl_up_sync(0xffffffffu, incl.h, o)};
        if ((int)lane >= o) incl = padd(incl, t);
    }
    const Pair total{__shfl_sync(0xffffffffu, incl.g, 31), __shfl_sync(0xffffffffu, incl.h, 31)};
    const bool reverse = !peq(total, sum);
    SplitRec mine;
    mine.flags = 0; mine.gain = 0.0f; mine.ord = 0xffffffffu; mine.bin = 0; mine.feat = f;
    mine.left = Pair{0, 0}; mine.right = Pair{0, 0};
    Pair run = psub(incl, loc);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t bidx = b0 + k;
        if (bidx < nb) {
            const Pair excl = run;
            run = padd(run, v[k]);
            float gain;
            const Pair r = psub(sum, run);
            if (split_gain(parent_gain, run, r, cons, ni.lower, ni.upper, sp, gain))
                consider(mine, gain, bidx, bidx + 1, 0u, run, r);
            if (reverse) {
                const Pair rr = psub(total, excl);
                const Pair ll = psub(sum, rr);
                if (split_gain(parent_gain, ll, rr, cons, ni.lower, ni.upper, sp, gain))
                    consider(mine, gain, nb + (nb - 1 - bidx), bidx, 2u, ll, rr);
            }
        }
    }
    // arg-max of (valid, gain, ordinal) over the warp; the lane holding the
    // winning ordinal writes its record (ordinals are unique per candidate)
    bool bv = (mine.flags & 1u) != 0;
    float bg = mine.gain;
    uint32_t bo = mine.ord;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const bool ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const float og = __shfl_xor_sync(0xffffffffu, bg, o);
        const uint32_t oo = __shfl_xor_sync(0xffffffffu, bo, o);
        if (ov && (!bv || og > bg || (og == bg && oo < bo))) { bv = true; bg = og; bo = oo; }
    }
    if (!bv) {
        if (lane == 0) *out = mine;  // flags 0
    } else if ((mine.flags & 1u) && mine.ord == bo) {
        *out = mine;
    }
}

// Per node: the best feature (equal gains -> lower feature id, split.rs:631-642).
// Last-block pattern for fusing a one-CTA step into the kernel before it:
// every CTA publishes its results, fences, and takes a ticket; the CTA that
// takes the last one (all others have finished) runs the step and resets
// the counter for the next launch.  No CTA waits on another.
__device__ __forceinline__ bool last_block_done(unsigned int* counter) {
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int ticket = atomicAdd(counter, 1u);
        last = ticket == gridDim.x - 1;
        if (last) *counter = 0u;
    }
    __syncthreads();
    if (last) __threadfence();
    return last;
}

__global__ void k_split_node(LevelArgs a) {
    const uint32_t node = blockIdx.x;
    if (node >= a.st->m) return;
    const uint32_t F = a.n_features, lane = threadIdx.x;
    float bg = 0.0f;
    uint32_t bf = 0xffffffffu;
    bool have = false;
    for (uint32_t f = a.feat_lo + lane; f < a.feat_hi; f += 32) {
        const SplitRec& r = a.feat_best[(size_t)node * F + f];
        if (!(r.flags & 1u)) continue;
        if (!have || r.gain > bg) { bg = r.gain; bf = f; have = true; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float og = __shfl_down_sync(0xffffffffu, bg, o);
        uint32_t of = __shfl_down_sync(0xffffffffu, bf, o);
        bool oh = __shfl_down_sync(0xffffffffu, (int)have, o);
        if (oh && (!have || og > bg || (og == bg && of < bf))) { bg = og; bf = of; have = true; }
    }
    have = __shfl_sync(0xffffffffu, (int)have, 0) != 0;
    bf = __shfl_sync(0xffffffffu, bf, 0);
    if (lane == 0) {
        SplitRec r;
        if (have) {
            r = a.feat_best[(size_t)node * F + bf];
            r.feat = bf;
        } else {
            r.flags = 0;
        }
        a.node_best[node] = r;
    }
    if (have && a.is_cat && a.is_cat[bf]) {
        const uint32_t W = a.cat_words;
        const uint32_t* src = a.feat_cats + ((size_t)node * a.n_cat + a.cat_slot[bf]) * W;
        for (uint32_t w = lane; w < W; w += 32) a.node_cats[(size_t)node * W + w] = src[w];
    }
}

// Depthwise decisions of one level (one CTA): the max_leaves budget in node
// order (training/mod.rs:4140-4151), tree arrays of the split nodes and their
// children (tree.rs:140-170 split_leaf; mod.rs:5069-5103 leaf values), and
// the children's sums / bounds.
template <int NT>
__device__ void decide_body(const LevelArgs& a, uint32_t* wt) {
    TreeState* st = a.st;
    const uint32_t m = st->m;
    const uint32_t leaf_count = st->leaf_count;
    const uint32_t base_nodes = st->n_tree_nodes;
    const uint32_t remaining = a.max_leaves == 0 ? 0xffffffffu
                                                 : (a.max_leaves > leaf_count ? a.max_leaves - leaf_count : 0u);
    const ScoreParams sp = load_sp(a);
    uint32_t found_before = 0;
    for (uint32_t c = 0; c < m; c += NT) {
        const uint32_t i = c + threadIdx.x;
        const bool found = i < m && (__ldcg(&a.node_best[i].flags) & 1u);
        uint32_t tot;
        const uint32_t rank = found_before + block_excl_scan_u32<NT>(found ? 1u : 0u, wt, tot);
        found_before += tot;
        if (i < m) {
            SplitDesc sd{-1, 0, 0, 0};
            if (found && rank < remaining) {
                SplitRec b;
                {
                    const uint4* src = reinterpret_cast<const uint4*>(&a.node_best[i]);
                    uint4* dst = reinterpret_cast<uint4*>(&b);
#pragma unroll
                    for (int q = 0; q < 4; q++) dst[q] = __ldcg(src + q);
                }
                const NodeInfo ni = a.nodes[i];
                const uint32_t k = rank;
                const int32_t L = (int32_t)(base_nodes + 2 * k), Rt = L + 1;
                const double lg = to_f64(b.left.g, sp.inv_g), lh = to_f64(b.left.h, sp.inv_h);
                const double rg = to_f64(b.right.g, sp.inv_g), rh = to_f64(b.right.h, sp.inv_h);
                const float wl = apply_bounds(xgb_weight(lg, lh, sp), ni.lower, ni.upper);
                const float wr = apply_bounds(xgb_weight(rg, rh, sp), ni.lower, ni.upper);
                const int cons = a.mono ? (int)a.mono[b.feat] : 0;
                const float mid = __fdiv_rn(__fadd_rn(wl, wr), 2.0f);
                float llo = ni.lower, lhi = ni.upper, rlo = ni.lower, rhi = ni.upper;
                if (cons < 0) { llo = mid; rhi = mid; } else if (cons > 0) { lhi = mid; rlo = mid; }
                const bool is_cat = (b.flags & 4u) != 0;
                TreeRec p;
                p.left = L; p.right = Rt; p.feat = b.feat; p.bin = b.bin; p.gain = b.gain; p.leaf = 0.0f;
                p.hess = a.trec[ni.tree_id].hess;
                p.flags = ((b.flags & 2u) ? 2u : 0u) | (is_cat ? 4u : 0u);
                a.trec[ni.tree_id] = p;  // a categorical node's set is in tcats already (k_split_node_decide)
                TreeRec cl{-1, -1, 0, 0, 0.0f, __fmul_rn(wl, sp.eta), __double2float_rn(lh), 1u};
                TreeRec cr{-1, -1, 0, 0, 0.0f, __fmul_rn(wr, sp.eta), __double2float_rn(rh), 1u};
                a.trec[L] = cl;
                a.trec[Rt] = cr;
                NodeInfo nl, nr;
                nl.tree_id = L; nl.sum = b.left; nl.lower = llo; nl.upper = lhi;
                nr.tree_id = Rt; nr.sum = b.right; nr.lower = rlo; nr.upper = rhi;
                nl.start = nr.start = 0; nl.len = nr.len = 0; nl.parent_slot = nr.parent_slot = -1;
                nl.acc_slot = nr.acc_slot = 0; nl.len_global = nr.len_global = 0;
                a.next_nodes[2 * k] = nl;
                a.next_nodes[2 * k + 1] = nr;
                sd.child_slot = (int32_t)(2 * k);
                sd.feat = b.feat;
                sd.bin = b.bin;
                sd.flags = b.flags & 6u;
            }
            a.split[i] = sd;
        }
    }
    if (threadIdx.x == 0) {
        const uint32_t kept = min(found_before, remaining);
        st->kept = kept;
        st->n_tree_nodes = base_nodes + 2 * kept;
        st->leaf_count = leaf_count + kept;
    }
}

// k_split_node for 8 nodes per CTA (one warp each) with the level's decisions
// (decide_body) run by the last CTA.
__global__ void __launch_bounds__(256) k_split_node_decide(LevelArgs a) {
    __shared__ uint32_t wt[32];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t node = blockIdx.x * 8 + warp;
    if (node < a.st->m) {
        const uint32_t F = a.n_features;
        float bg = 0.0f;
        uint32_t bf = 0xffffffffu;
        bool have = false;
        for (uint32_t f = a.feat_lo + lane; f < a.feat_hi; f += 32) {
            const SplitRec& r = a.feat_best[(size_t)node * F + f];
            if (!(r.flags & 1u)) continue;
            if (!have || r.gain > bg) { bg = r.gain; bf = f; have = true; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float og = __shfl_down_sync(0xffffffffu, bg, o);
            uint32_t of = __shfl_down_sync(0xffffffffu, bf, o);
            bool oh = __shfl_down_sync(0xffffffffu, (int)have, o);
            if (oh && (!have || og > bg || (og == bg && of < bf))) { bg = og; bf = of; have = true; }
        }
        have = __shfl_sync(0xffffffffu, (int)have, 0) != 0;
        bf = __shfl_sync(0xffffffffu, bf, 0);
        if (lane == 0) {
            SplitRec r;
            if (have) {
                r = a.feat_best[(size_t)node * F + bf];
                r.feat = bf;
            } else {
                r.flags = 0;
            }
            a.node_best[node] = r;
        }
        if (have && a.is_cat && a.is_cat[bf]) {
            // the set goes to the node's tree record too (read only if decide_body splits the node)
            const uint32_t W = a.cat_words;
            const uint32_t* src = a.feat_cats + ((size_t)node * a.n_cat + a.cat_slot[bf]) * W;
            const size_t tid = (size_t)a.nodes[node].tree_id;
            for (uint32_t w = lane; w < W; w += 32) {
                const uint32_t v = src[w];
                a.node_cats[(size_t)node * W + w] = v;
                a.tcats[tid * W + w] = v;
            }
        }
    }
    if (last_block_done(a.fuse + 0)) decide_body<256>(a, wt);
}

// Feature-sharded split search of a row-sharded run: each rank's per-node
// winner over its own features (k_split_node), gathered in rank order, is
// merged into the node's best split.  A strictly greater gain replaces the
// current winner, so equal gains keep the lower rank's, which is the lower
// feature (ranks own ascending feature ranges; split.rs:631-642).  The
// winner's category set goes to the node and its tree record, then the last
// CTA runs the level's decisions.
__global__ void __launch_bounds__(256) k_merge_decide(LevelArgs a, const SplitRec* __restrict__ all_best,
                                                      const uint32_t* __restrict__ all_cats, uint32_t n_ranks,
                                                      uint32_t stride) {
    __shared__ uint32_t wt[32];
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.st->m) {
        int best = -1;
        float bg = 0.0f;
        for (uint32_t r = 0; r < n_ranks; r++) {
            const SplitRec& rec = all_best[(size_t)r * stride + i];
            if (!(rec.flags & 1u)) continue;
            if (best < 0 || rec.gain > bg) { best = (int)r; bg = rec.gain; }
        }
        SplitRec out;
        if (best >= 0) {
            out = all_best[(size_t)best * stride + i];
        } else {
            out.flags = 0;
        }
        a.node_best[i] = out;
        if (best >= 0 && (out.flags & 4u)) {
            const uint32_t W = a.cat_words;
            const uint32_t* src = all_cats + ((size_t)best * stride + i) * W;
            const size_t tid = (size_t)a.nodes[i].tree_id;
            for (uint32_t w = 0; w < W; w++) {
                a.node_cats[(size_t)i * W + w] = src[w];
                a.tcats[tid * W + w] = src[w];
            }
        }
    }
    if (last_block_done(a.fuse + 0)) decide_body<256>(a, wt);
}

// ------------------------------------------------------------------ partition
// categorical.rs:330-345: a code in the set goes right; codes beyond the set's words go left
__device__ __forceinline__ bool cat_left(const uint32_t* cats, uint32_t words, uint32_t bin) {
    return bin >= 32u * words || ((cats[bin >> 5] >> (bin & 31)) & 1u) == 0u;
}

__device__ __forceinline__ bool goes_left(const LevelArgs& a, const SplitDesc& sd, const uint32_t* cats,
                                          uint32_t row) {
    const FeatLoc fl = a.floc[sd.feat];
    const uint8_t* p = fl.base + (size_t)row * fl.stride + fl.byte_off;
    uint32_t bin = fl.width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
    if (bin == fl.missing) return (sd.flags & 2u) != 0;
    if (sd.flags & 4u) return cat_left(cats, a.cat_words, bin);
    return bin < sd.bin;
}

// The category set of node j of the level: copied to shared memory when it
// is the usual 8 words (cats_s), else read in place.
__device__ __forceinline__ const uint32_t* node_set(const LevelArgs& a, uint32_t j, uint32_t* cats_s) {
    const uint32_t* g = a.node_cats + (size_t)j * a.cat_words;
    if (a.cat_words != 8u) return g;
    if (threadIdx.x < 8) cats_s[threadIdx.x] = g[threadIdx.x];
    return cats_s;
}

// Count the left rows of every chunk of a split node; add the leaf value to
// the predictions of every row of a node that stops growing here
// (training/mod.rs:4409-4425; delta[row] = leaf, then pred += delta, is the
// same single f32 addition).  Thread t owns rows [8t, 8t + 8) of its chunk;
// with a.dirflags set it stores their directions as one byte (bit k = row
// 8t + k goes left) so the scatter pass does not gather the bins again.
__device__ __forceinline__ void part_count_work(const LevelArgs& a) {
    __shared__ uint32_t wt[32];
    __shared__ uint32_t cats[8];
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t m = st->m;
    const uint32_t j = find_segment_warp(a.chunk_prefix, m, c);
    const NodeInfo ni = a.nodes[j];
    const uint32_t r0 = (c - a.chunk_prefix[j]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* rows = a.rows_cur + ni.start + r0;
    const SplitDesc sd = a.split[j];
    const uint32_t i0 = threadIdx.x * kPartItems;
    uint32_t r[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) r[k] = i0 + k < cnt ? rows[i0 + k] : 0u;
    if (sd.child_slot < 0) {
        if (!a.walk) {  // with k_tree_walk the leaf reaches these rows after the tree is finished
            const float leaf = a.trec[ni.tree_id].leaf;
#pragma unroll
            for (int k = 0; k < kPartItems; k++)
                if (i0 + k < cnt) a.pred[r[k]] = __fadd_rn(a.pred[r[k]], leaf);
        }
        if (threadIdx.x == 0) a.chunk_left[c] = 0u;
        return;
    }
    const uint32_t* set = node_set(a, j, cats);
    const FeatLoc fl = a.floc[sd.feat];
    __syncthreads();
    uint32_t bin[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        bin[k] = fl.missing;
        if (i0 + k < cnt) {
            const uint8_t* p = fl.base + (size_t)r[k] * fl.stride + fl.byte_off;
            bin[k] = fl.width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
        }
    }
    uint32_t flags = 0;
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        bool left;
        if (bin[k] == fl.missing) left = (sd.flags & 2u) != 0;
        else if (sd.flags & 4u) left = cat_left(set, a.cat_words, bin[k]);
        else left = bin[k] < sd.bin;
        if (i0 + k < cnt && left) flags |= 1u << k;
    }
    if (a.dirflags) a.dirflags[(size_t)c * kPartThreads + threadIdx.x] = (uint8_t)flags;
    uint32_t tot;
    (void)block_excl_scan_u32<kPartThreads>((uint32_t)__popc(flags), wt, tot);
    if (threadIdx.x == 0) a.chunk_left[c] = tot;
}

// Exclusive scan of the chunk left counts (one CTA) and per-node left totals.
template <int NT>
__device__ void part_scan_body(const LevelArgs& a, uint32_t* wt) {
    const TreeState* st = a.st;
    const uint32_t nc = st->chunk_count, m = st->m;
    uint32_t carry = 0;
    for (uint32_t base = 0; base < nc; base += NT) {
        const uint32_t c = base + threadIdx.x;
        const uint32_t v = c < nc ? __ldcg(&a.chunk_left[c]) : 0u;
        uint32_t tot;
        const uint32_t ex = block_excl_scan_u32<NT>(v, wt, tot);
        if (c < nc) a.chunk_off[c] = carry + ex;
        carry += tot;
    }
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < m; j += blockDim.x) {
        const uint32_t c0 = a.chunk_prefix[j], c1 = a.chunk_prefix[j + 1];
        const uint32_t first = c0 < nc ? a.chunk_off[c0] : carry;
        const uint32_t last = c1 < nc ? a.chunk_off[c1] : carry;
        a.node_left[j] = last - first;
    }
}

__global__ void __launch_bounds__(1024) k_part_scan(LevelArgs a) {
    __shared__ uint32_t wt[32];
    part_scan_body<1024>(a, wt);
}

// Stable scatter of every chunk of a split node into [left | right] of the
// node's span in the next arena (directions from k_part_count's bytes, or
// recomputed when a.dirflags is null).
__device__ __forceinline__ void part_scatter_work(const LevelArgs& a) {
    __shared__ uint32_t wt[32];
    __shared__ uint32_t cats[8];
    __shared__ uint32_t stage[kChunkRows];
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t m = st->m;
    const uint32_t j = find_segment_warp(a.chunk_prefix, m, c);
    const SplitDesc sd = a.split[j];
    if (sd.child_slot < 0) return;
    const NodeInfo ni = a.nodes[j];
    const uint32_t r0 = (c - a.chunk_prefix[j]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* rows = a.rows_cur + ni.start + r0;
    const uint32_t i0 = threadIdx.x * kPartItems;
    uint32_t r[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) r[k] = i0 + k < cnt ? rows[i0 + k] : 0u;
    uint32_t flags = 0;
    if (a.dirflags) {
        flags = a.dirflags[(size_t)c * kPartThreads + threadIdx.x];
    } else {
        const uint32_t* set = node_set(a, j, cats);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kPartItems; k++)
            if (i0 + k < cnt && goes_left(a, sd, set, r[k])) flags |= 1u << k;
    }
    const uint32_t nl = (uint32_t)__popc(flags);
    uint32_t L;
    const uint32_t lpos = block_excl_scan_u32<kPartThreads>(nl, wt, L);
    uint32_t li = lpos, ri = L + (min(i0, cnt) - lpos);
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        const uint32_t i = i0 + k;
        if (i < cnt) {
            if (flags & (1u << k)) stage[li++] = r[k];
            else stage[ri++] = r[k];
        }
    }
    __syncthreads();
    const uint32_t node_first = a.chunk_off[a.chunk_prefix[j]];
    const uint32_t left_before = a.chunk_off[c] - node_first;
    const uint32_t right_before = r0 - left_before;
    const uint32_t node_nl = a.node_left[j];
    uint32_t* dst_l = a.rows_next + ni.start + left_before;
    uint32_t* dst_r = a.rows_next + ni.start + node_nl + right_before;
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        if (i < L) dst_l[i] = stage[i];
        else dst_r[i - L] = stage[i];
    }
}

// Next level's node table, accumulate list and chunk table (one CTA).  The
// smaller child (by rows, training/mod.rs:4478-4482; by hessian sum over all
// ranks when row-sharded) is accumulated, the larger one is its parent minus
// the smaller one.  Which one is accumulated never changes the histograms.
template <int NT>
__device__ void next_level_body(const LevelArgs& a, unsigned long long* wt64, uint32_t* wt) {
    TreeState* st = a.st;
    const uint32_t m = st->m, kept = st->kept;
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
        const SplitDesc sd = a.split[i];
        if (sd.child_slot < 0) continue;
        const uint32_t k = (uint32_t)sd.child_slot >> 1;
        const NodeInfo ni = a.nodes[i];
        const uint32_t nl = a.node_left[i], nr = ni.len - nl;
        NodeInfo& L = a.next_nodes[2 * k];
        NodeInfo& R = a.next_nodes[2 * k + 1];
        L.start = ni.start; L.len = nl;
        R.start = ni.start + nl; R.len = nr;
        uint32_t small;
        if (a.node_left_global) {
            const uint32_t nlg = a.node_left_global[i], nrg = ni.len_global - nlg;
            L.len_global = nlg; R.len_global = nrg;
            small = nlg <= nrg ? 0u : 1u;
        } else {  // row-sharded: by the children's global hessian sums
            L.len_global = R.len_global = 0;
            small = L.sum.h <= R.sum.h ? 0u : 1u;
        }
        L.acc_slot = (int32_t)k; R.acc_slot = (int32_t)k;
        L.parent_slot = small == 0 ? -1 : (int32_t)i;
        R.parent_slot = small == 1 ? -1 : (int32_t)i;
        a.next_acc_list[k] = 2 * k + small;
    }
    __syncthreads();
    unsigned long long carry = 0;
    for (uint32_t base = 0; base < kept; base += NT) {
        const uint32_t k = base + threadIdx.x;
        unsigned long long v = k < kept ? a.next_nodes[a.next_acc_list[k]].len : 0ull;
        unsigned long long tot;
        unsigned long long ex = block_excl_scan_u64<NT>(v, wt64, tot);
        if (k < kept) a.next_acc_prefix[k] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) a.next_acc_prefix[kept] = carry;
    uint32_t ccarry = 0;
    const uint32_t m2 = 2 * kept;
    for (uint32_t base = 0; base < m2; base += NT) {
        const uint32_t s = base + threadIdx.x;
        const uint32_t v = s < m2 ? (a.next_nodes[s].len + kChunkRows - 1) / kChunkRows : 0u;
        uint32_t tot;
        const uint32_t ex = block_excl_scan_u32<NT>(v, wt, tot);
        if (s < m2) a.next_chunk_prefix[s] = ccarry + ex;
        ccarry += tot;
    }
    if (threadIdx.x == 0) {
        a.next_chunk_prefix[m2] = ccarry;
        st->m = m2;
        st->acc_count = kept;
        st->acc_total = carry;
        st->chunk_count = ccarry;
    }
}

// Stable partition passes (count, k_part_scan, scatter): the single-node
// partition entry points and lossguide growth.
__global__ void __launch_bounds__(kPartThreads) k_part_count(LevelArgs a) { part_count_work(a); }

__global__ void __launch_bounds__(kPartThreads) k_part_scatter(LevelArgs a) { part_scatter_work(a); }

// Depthwise growth: the whole level partition in one pass.  Each chunk CTA
// finds its rows' directions, reserves room with one 64-bit atomic on its
// node's counter pair (left rows counted up from the node's start in the low
// word, right rows counted down from its end in the high word; a node holds
// fewer than 2^32 rows, so the low word never carries) and writes its rows
// there in row order.  Chunks of one node land in the order their
// reservations happen, so a child's span is a run of row-ordered pieces
// rather than one row-ordered run: nothing downstream depends on the order
// (histograms are exact integer sums, leaf values are added per row, the
// child sizes are the same).  Rows of nodes that stop growing get their leaf
// value as in k_part_count.
__device__ __forceinline__ void part_level_work(const LevelArgs& a) {
    __shared__ uint32_t wt[32];
    __shared__ uint32_t cats[8];
    __shared__ uint32_t stage[kChunkRows];
    __shared__ unsigned long long base;
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t m = st->m;
    const uint32_t j = find_segment_warp(a.chunk_prefix, m, c);
    const NodeInfo ni = a.nodes[j];
    const uint32_t r0 = (c - a.chunk_prefix[j]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* rows = a.rows_cur + ni.start + r0;
    const SplitDesc sd = a.split[j];
    const uint32_t i0 = threadIdx.x * kPartItems;
    uint32_t r[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) r[k] = i0 + k < cnt ? rows[i0 + k] : 0u;
    if (sd.child_slot < 0) {
        if (!a.walk) {
            const float leaf = a.trec[ni.tree_id].leaf;
#pragma unroll
            for (int k = 0; k < kPartItems; k++)
                if (i0 + k < cnt) a.pred[r[k]] = __fadd_rn(a.pred[r[k]], leaf);
        }
        return;
    }
    const uint32_t* set = node_set(a, j, cats);
    const FeatLoc fl = a.floc[sd.feat];
    __syncthreads();
    uint32_t flags = 0;
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        uint32_t bin = fl.missing;
        if (i0 + k < cnt) {
            const uint8_t* p = fl.base + (size_t)r[k] * fl.stride + fl.byte_off;
            bin = fl.width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
        }
        bool left;
        if (bin == fl.missing) left = (sd.flags & 2u) != 0;
        else if (sd.flags & 4u) left = cat_left(set, a.cat_words, bin);
        else left = bin < sd.bin;
        if (i0 + k < cnt && left) flags |= 1u << k;
    }
    uint32_t L;
    const uint32_t lpos = block_excl_scan_u32<kPartThreads>((uint32_t)__popc(flags), wt, L);
    if (threadIdx.x == 0)
        base = atomicAdd(&a.part_cnt[j], (unsigned long long)L | ((unsigned long long)(cnt - L) << 32));
    uint32_t li = lpos, ri = L + (min(i0, cnt) - lpos);
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        if (i0 + k < cnt) {
            if (flags & (1u << k)) stage[li++] = r[k];
            else stage[ri++] = r[k];
        }
    }
    __syncthreads();
    const uint32_t lbase = (uint32_t)base, rbase = (uint32_t)(base >> 32);
    uint32_t* dst_l = a.rows_next + ni.start + lbase;
    // this chunk's right rows end where the rows reserved before them begin
    uint32_t* dst_r = a.rows_next + ni.start + (ni.len - rbase - (cnt - L));
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        if (i < L) dst_l[i] = stage[i];
        else dst_r[i - L] = stage[i];
    }
}

// The last CTA turns the counter pairs into the per-node left counts, clears
// them for the next level and builds the next level (next_level_body).  At
// 32 registers four 512-thread CTAs fit an SM (three at the 40 the compiler
// takes unbounded): the pass waits on its dependent loads, so residency is
// what hides them.
__global__ void __launch_bounds__(kPartThreads, 4) k_part_level(LevelArgs a) {
    // the next level's accumulate histograms, read by this level's split
    // search (finished before this kernel) and not again, start at zero
    if (a.hist_zero) {
        uint4* z = reinterpret_cast<uint4*>(a.hist_zero);
        const unsigned long long n16 = a.hist_zero_words / 2;
        for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
             i += (unsigned long long)gridDim.x * blockDim.x)
            z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    part_level_work(a);
    if (last_block_done(a.fuse + 1)) {
        __shared__ unsigned long long wt64_next[32];
        __shared__ uint32_t wt_next[32];
        const uint32_t m = a.st->m;
        for (uint32_t j = threadIdx.x; j < m; j += blockDim.x) {
            a.node_left[j] = (uint32_t)__ldcg(&a.part_cnt[j]);
            a.part_cnt[j] = 0ull;
        }
        __syncthreads();
        next_level_body<kPartThreads>(a, wt64_next, wt_next);
    }
}

// Depthwise, the last level without the tree walk: the children are final
// leaves, so each row's leaf value goes to its margin here instead of after a
// partition into the children (k_part_level, then k_leaf_final): a row of a
// split node takes its child's value (the same direction test as
// k_part_level), a row of a node that stops here takes the node's own.  One
// f32 addition per row, as on the other path; no row is written.
__global__ void __launch_bounds__(kPartThreads) k_part_final(LevelArgs a) {
    __shared__ uint32_t cats[8];
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t j = find_segment_warp(a.chunk_prefix, st->m, c);
    const NodeInfo ni = a.nodes[j];
    const uint32_t r0 = (c - a.chunk_prefix[j]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* rows = a.rows_cur + ni.start + r0;
    const SplitDesc sd = a.split[j];
    const uint32_t i0 = threadIdx.x * kPartItems;
    uint32_t r[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) r[k] = i0 + k < cnt ? rows[i0 + k] : 0u;
    if (sd.child_slot < 0) {
        const float leaf = a.trec[ni.tree_id].leaf;
#pragma unroll
        for (int k = 0; k < kPartItems; k++)
            if (i0 + k < cnt) a.pred[r[k]] = __fadd_rn(a.pred[r[k]], leaf);
        return;
    }
    const uint32_t* set = node_set(a, j, cats);
    const FeatLoc fl = a.floc[sd.feat];
    const float leaf_l = a.trec[a.next_nodes[sd.child_slot].tree_id].leaf;
    const float leaf_r = a.trec[a.next_nodes[sd.child_slot + 1].tree_id].leaf;
    __syncthreads();
    uint32_t bin[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        bin[k] = fl.missing;
        if (i0 + k < cnt) {
            const uint8_t* p = fl.base + (size_t)r[k] * fl.stride + fl.byte_off;
            bin[k] = fl.width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
        }
    }
    float pv[kPartItems];
#pragma unroll
    for (int k = 0; k < kPartItems; k++) pv[k] = i0 + k < cnt ? a.pred[r[k]] : 0.0f;
#pragma unroll
    for (int k = 0; k < kPartItems; k++) {
        bool left;
        if (bin[k] == fl.missing) left = (sd.flags & 2u) != 0;
        else if (sd.flags & 4u) left = cat_left(set, a.cat_words, bin[k]);
        else left = bin[k] < sd.bin;
        if (i0 + k < cnt) a.pred[r[k]] = __fadd_rn(pv[k], left ? leaf_l : leaf_r);
    }
}

// Final level: every remaining node is a leaf (training/mod.rs:4524-4550).
__global__ void __launch_bounds__(kPartThreads) k_leaf_final(LevelArgs a) {
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t j = find_segment_warp(a.chunk_prefix, st->m, c);
    const NodeInfo ni = a.nodes[j];
    const uint32_t r0 = (c - a.chunk_prefix[j]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* rows = a.rows_cur + ni.start + r0;
    const float leaf = a.trec[ni.tree_id].leaf;
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        const uint32_t r = rows[i];
        a.pred[r] = __fadd_rn(a.pred[r], leaf);
    }
}

// One thread per row, rows in order so the margin update is coalesced: from
// the root, each split reads the row's bin of its feature and goes the way
// the partition would (missing -> default direction, categorical set ->
// right, else bin < split bin -> left); the leaf's value is added to the
// row's margin.  Trees of up to kWalkNodes nodes are first laid out in shared
// memory, one 32-byte entry per node holding everything a step needs.  When
// all features sit in one record block of at most kWalkStageBytes per row
// (a.walk_rec), each CTA first copies its 256 rows' records into shared
// memory with coalesced word loads (pitch + 4 bytes, so the 32 lanes' rows
// fall in different banks) and the steps read bins from there; otherwise each
// step reads its byte from the records in global memory.
constexpr uint32_t kWalkThreads = 256;
constexpr uint32_t kWalkStageBytes = 64;
// One 16-byte entry per node, read with one shared load per step.
struct alignas(16) WalkNode {
    uint32_t lr;       // split: left | right << 16 (tree-local ids)
    uint32_t bin_fl;   // split bin | node flags << 16 | bin width << 24
    uint32_t val;      // split: missing sentinel; leaf: the leaf value's bits
    uint32_t loc;      // split: the feature's byte offset in the staged record, or its id (unstaged)
};
static_assert(sizeof(WalkNode) == 16, "WalkNode layout");

// WORDS: 32-bit words staged per row (records of up to 4 * WORDS bytes).
// GRAD: the walk also computes the next round's gradient pairs from the new
// margins (what k_gradient_max would compute at the start of that round, in
// mode gmode: 1 fexp_core alone, 2 the host expf reproduced) and folds their
// bounds into ga.maxbits, so that round starts at its scales.
template <uint32_t WORDS, bool GRAD>
__global__ void __launch_bounds__(kWalkThreads) k_tree_walk(LevelArgs a, uint32_t n_rows, GradArgs ga, int gmode) {
    __shared__ WalkNode wn[kWalkNodes];
    __shared__ uint32_t stage[kWalkThreads * (WORDS + 1)];
    __shared__ uint32_t plain;  // every split numeric on one-byte bins, right child = left + 1
    const uint32_t nn = a.st->n_tree_nodes;
    const bool table = nn <= kWalkNodes;
    const bool staged = table && a.walk_rec != nullptr;
    if (threadIdx.x == 0) plain = 1u;
    __syncthreads();
    if (table) {
        for (uint32_t i = threadIdx.x; i < nn; i += blockDim.x) {
            const TreeRec t = a.trec[i];
            WalkNode w{};
            if (t.flags & 1u) {
                w.bin_fl = 1u << 16;
                w.val = __float_as_uint(t.leaf);
            } else {
                const FeatLoc fl = a.floc_rec[t.feat];
                w.lr = (uint32_t)t.left | ((uint32_t)t.right << 16);
                w.bin_fl = (t.bin & 0xffffu) | ((t.flags & 0xffu) << 16) | (fl.width << 24);
                w.val = fl.missing;
                w.loc = staged ? fl.byte_off : t.feat;
                if ((t.flags & 4u) || fl.width != 1 || t.right != t.left + 1) plain = 0u;
            }
            wn[i] = w;
        }
    }
    const uint32_t words = a.walk_stride / 4, pitch = words + 1;
    const uint8_t* srow = reinterpret_cast<const uint8_t*>(stage + threadIdx.x * pitch);
    // staged: the next step's records are loaded into registers (word i of
    // the step's contiguous block at i = threadIdx.x + k * blockDim.x) while
    // the current step walks, then stored to shared memory
    constexpr uint32_t kWalkWords = WORDS;
    uint32_t nxt[kWalkWords];
    const uint32_t step = blockDim.x * gridDim.x;
    auto load_next = [&](uint32_t base) {
        const uint32_t rows = base < n_rows ? min((uint32_t)blockDim.x, n_rows - base) : 0u;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(a.walk_rec + (size_t)base * a.walk_stride);
#pragma unroll
        for (uint32_t k = 0; k < kWalkWords; k++) {
            const uint32_t i = threadIdx.x + k * blockDim.x;
            nxt[k] = (k < words && i < rows * words) ? src[i] : 0u;
        }
    };
    auto store_next = [&]() {
        if (words == kWalkWords) {  // records of exactly kWalkWords words: no runtime division
#pragma unroll
            for (uint32_t k = 0; k < kWalkWords; k++) {
                const uint32_t i = threadIdx.x + k * blockDim.x;
                stage[(i / kWalkWords) * (kWalkWords + 1) + i % kWalkWords] = nxt[k];
            }
            return;
        }
#pragma unroll
        for (uint32_t k = 0; k < kWalkWords; k++) {
            const uint32_t i = threadIdx.x + k * blockDim.x;
            if (k < words) {
                const uint32_t rr = i / words, ww = i - rr * words;
                stage[rr * pitch + ww] = nxt[k];
            }
        }
    };
    if (staged) load_next(blockIdx.x * blockDim.x);
    __syncthreads();
    // the common tree: one 16-byte node load, one staged byte, a compare and
    // an add per level
    const bool fast = staged && plain != 0u;
    const uint4* wn4 = reinterpret_cast<const uint4*>(wn);
    double mg = 0.0, mh = 0.0;  // GRAD: bounds of this thread's gradient pairs
    auto next_gradient = [&](uint32_t r, float m) {
        float e = 0.0f;
        if (ga.objective == 1) {
            const float x = -m;
            e = gmode == 2 ? host_expf(x, ga.exptab, ga.exp_probes) : fbx::fexp_core(x);
        }
        float g, h;
        row_gradient_m(ga, r, e, m, g, h);
        reinterpret_cast<float2*>(ga.gpair_f32)[r] = make_float2(g, h);
        mg = fmax(mg, bound_of(g));
        mh = fmax(mh, bound_of(h));
    };
    for (uint32_t base = blockIdx.x * blockDim.x; base < n_rows; base += step) {
        const uint32_t r = base + threadIdx.x;
        if (staged) {
            store_next();
            __syncthreads();
            load_next(base + step);
        }
        const float pv = r < n_rows ? a.pred[r] : 0.0f;  // in flight during the walk
        if (fast) {
            if (r < n_rows) {
                uint4 q = wn4[0];
                for (uint32_t depth = 0; depth < 64 && !(q.y & (1u << 16)); depth++) {
                    const uint32_t bin = srow[q.w];
                    const bool left = bin == q.z ? (q.y & (2u << 16)) != 0u : bin < (q.y & 0xffffu);
                    q = wn4[(q.x & 0xffffu) + (left ? 0u : 1u)];
                }
                float m = pv;
                if (q.y & (1u << 16)) {
                    m = __fadd_rn(pv, __uint_as_float(q.z));
                    a.pred[r] = m;
                }
                if (GRAD) next_gradient(r, m);
            }
        } else if (r < n_rows) {
            float m = pv;
            uint32_t node = 0;
            for (uint32_t depth = 0; depth < 64; depth++) {  // trees are at most 15 levels deep
                uint32_t flags, sbin, missing, width, left_id, right_id, bin;
                float leaf = 0.0f;
                if (table) {
                    const uint4 q = wn4[node];
                    const WalkNode w{q.x, q.y, q.z, q.w};
                    flags = (w.bin_fl >> 16) & 0xffu;
                    if (flags & 1u) leaf = __uint_as_float(w.val);
                    sbin = w.bin_fl & 0xffffu;
                    width = w.bin_fl >> 24;
                    missing = w.val;
                    left_id = w.lr & 0xffffu;
                    right_id = w.lr >> 16;
                    if (!(flags & 1u)) {
                        if (staged) {
                            bin = width == 2 ? (uint32_t)srow[w.loc] | ((uint32_t)srow[w.loc + 1] << 8)
                                             : (uint32_t)srow[w.loc];
                        } else {
                            const FeatLoc fl = a.floc_rec[w.loc];
                            const uint8_t* p = fl.base + (size_t)r * fl.stride + fl.byte_off;
                            bin = width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
                        }
                    }
                } else {
                    const TreeRec t = a.trec[node];
                    flags = t.flags;
                    leaf = t.leaf;
                    sbin = t.bin;
                    left_id = (uint32_t)t.left;
                    right_id = (uint32_t)t.right;
                    if (!(flags & 1u)) {
                        const FeatLoc fl = a.floc_rec[t.feat];
                        width = fl.width;
                        missing = fl.missing;
                        const uint8_t* p = fl.base + (size_t)r * fl.stride + fl.byte_off;
                        bin = width == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(p) : (uint32_t)*p;
                    }
                }
                if (flags & 1u) {
                    m = __fadd_rn(pv, leaf);
                    a.pred[r] = m;
                    break;
                }
                bool left;
                if (bin == missing) left = (flags & 2u) != 0;
                else if (flags & 4u) left = cat_left(a.tcats + (size_t)node * a.cat_words, a.cat_words, bin);
                else left = bin < sbin;
                node = left ? left_id : right_id;
            }
            if (GRAD) next_gradient(r, m);
        }
        if (staged) __syncthreads();
    }
    if (GRAD) fold_max(mg, mh, ga.maxbits);
}

// Root of a new tree (training/mod.rs:3466-3469, 3499-3501).
__global__ void k_tree_init(LevelArgs a, uint32_t n_local, uint32_t n_global, const unsigned long long* root_sum) {
    if (threadIdx.x != 0) return;
    const Pair sum{(long long)root_sum[0], (long long)root_sum[1]};
    NodeInfo r;
    r.start = 0; r.len = n_local; r.tree_id = 0; r.parent_slot = -1; r.acc_slot = 0;
    r.lower = -FLT_MAX; r.upper = FLT_MAX; r.len_global = n_global; r.sum = sum;
    a.nodes[0] = r;
    const ScoreParams sp = load_sp(a);
    const double g = to_f64(sum.g, sp.inv_g), h = to_f64(sum.h, sp.inv_h);
    TreeRec t{-1, -1, 0, 0, 0.0f, __fmul_rn(xgb_weight(g, h, sp), sp.eta), __double2float_rn(h), 1u};
    a.trec[0] = t;
    const_cast<uint32_t*>(a.acc_list)[0] = 0;
    const_cast<unsigned long long*>(a.acc_prefix)[0] = 0;
    const_cast<unsigned long long*>(a.acc_prefix)[1] = n_local;
    const_cast<uint32_t*>(a.chunk_prefix)[0] = 0;
    const_cast<uint32_t*>(a.chunk_prefix)[1] = (n_local + kChunkRows - 1) / kChunkRows;
    TreeState* st = a.st;
    st->m = 1; st->n_tree_nodes = 1; st->leaf_count = 1; st->acc_count = 1; st->acc_total = n_local;
    st->chunk_count = (n_local + kChunkRows - 1) / kChunkRows; st->kept = 0; st->error = 0;
    st->rank_stride = 0;
}

__global__ void k_iota(uint32_t* rows, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += blockDim.x * gridDim.x) rows[i] = i;
}

// Column-major block (reference BinData, columns.rs:9-25) to the device's
// row-major record layout: dst[row * stride + local * width].
template <int W>
__global__ void k_transpose_block(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t n_rows,
                                  uint32_t n_feats, uint32_t stride, uint64_t row0) {
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < (uint64_t)n_rows * n_feats;
         idx += (uint64_t)blockDim.x * gridDim.x) {
        const uint32_t f = (uint32_t)(idx / n_rows);
        const uint32_t r = (uint32_t)(idx % n_rows);
        if (W == 2) {
            const uint16_t v = reinterpret_cast<const uint16_t*>(src)[(size_t)f * n_rows + r];
            *reinterpret_cast<uint16_t*>(dst + (size_t)(row0 + r) * stride + (size_t)f * 2) = v;
        } else {
            dst[(size_t)(row0 + r) * stride + f] = src[(size_t)f * n_rows + r];
        }
    }
}

// Column-major copy of a block's row records (feature i of the block at
// cols + i * n_rows * W): the partition passes gather one bin per row, and
// the rows of a node come in runs of ascending ids, so at the shallow levels
// neighbouring rows of a node share the 32-byte sectors of a column but never
// a record's.
// Tiled transpose: a CTA stages kTrRows records in shared memory with
// coalesced word loads (row pitch stride + 4 bytes, so the column reads hit
// distinct banks), then writes each feature's kTrRows bins contiguously.
constexpr uint32_t kTrRows = 256;
template <int W>
__global__ void __launch_bounds__(256) k_records_to_columns(const uint8_t* __restrict__ rec, uint32_t stride,
                                                            uint64_t n_rows, uint32_t n_feats,
                                                            uint8_t* __restrict__ cols) {
    extern __shared__ uint32_t tile[];
    const uint32_t wpr = stride / 4, pitch = wpr + 1;  // words per record, padded pitch
    for (uint64_t r0 = (uint64_t)blockIdx.x * kTrRows; r0 < n_rows; r0 += (uint64_t)gridDim.x * kTrRows) {
        const uint32_t rows = (uint32_t)min((uint64_t)kTrRows, n_rows - r0);
        const uint32_t* src = reinterpret_cast<const uint32_t*>(rec + r0 * stride);
        for (uint32_t i = threadIdx.x; i < rows * wpr; i += blockDim.x) {
            const uint32_t r = i / wpr, w = i - r * wpr;
            tile[r * pitch + w] = src[i];
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < rows * n_feats; i += blockDim.x) {
            const uint32_t f = i / rows, r = i - f * rows;
            const uint8_t* row = reinterpret_cast<const uint8_t*>(tile + r * pitch);
            if (W == 2)
                reinterpret_cast<uint16_t*>(cols)[f * n_rows + r0 + r] = *reinterpret_cast<const uint16_t*>(row + f * 2);
            else
                cols[f * n_rows + r0 + r] = row[f];
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ launchers
// CTAs of `threads` threads (static shared memory only) that the device's
// SMs hold at once for `kernel` (a failed query gives one CTA per SM of a
// B200: a smaller grid, never a wrong result; the launch reports the error).
static uint32_t resident_grid(const void* kernel, uint32_t threads) {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, (int)threads, 0) != cudaSuccess || per_sm <= 0)
        per_sm = 1;
    return (uint32_t)(sms * per_sm);
}

static unsigned grad_grid(uint32_t n) {
    unsigned b = (n + 255) / 256;
    return b < 148u * 8u ? (b ? b : 1u) : 148u * 8u;
}
void launch_mask_max(const GradArgs& a, cudaStream_t s) { count_launch(); k_mask_max<<<grad_grid(a.n), 256, 0, s>>>(a); }
void launch_gradient_max(const GradArgs& a, int mode, cudaStream_t s) {
    count_launch();
    k_gradient_max<<<grad_grid(a.n), 256, 0, s>>>(a, mode);
}
void launch_expf_emulate(const uint2* tab, uint32_t probes, uint32_t begin, uint32_t count, uint32_t* out,
                         cudaStream_t s) {
    count_launch();
    k_expf_emulate<<<148 * 8, 256, 0, s>>>(tab, probes, begin, count, out);
}
void launch_gradient_quantize_exp(const GradArgs& a, cudaStream_t s) {
    count_launch();
    k_gradient_quantize_exp<<<grad_grid(a.n), 256, 0, s>>>(a);
}
void launch_quantize(const GradArgs& a, cudaStream_t s) { count_launch(); k_quantize<<<grad_grid(a.n), 256, 0, s>>>(a); }
void launch_softmax_gradients(const GradArgs& a, uint32_t K, float* out, int fast, cudaStream_t s) {
    count_launch();
    if (K <= 16) {
        if (fast)
            k_softmax_grad<true, 16><<<grad_grid(a.n), 256, 0, s>>>(a, K, out);
        else
            k_softmax_grad<false, 16><<<grad_grid(a.n), 256, 0, s>>>(a, K, out);
    } else {
        if (fast)
            k_softmax_grad<true, 0><<<grad_grid(a.n), 256, 0, s>>>(a, K, out);
        else
            k_softmax_grad<false, 0><<<grad_grid(a.n), 256, 0, s>>>(a, K, out);
    }
}
void launch_device_scales(const unsigned long long* maxbits, unsigned long long n_rows, double* scales,
                          unsigned long long* err, cudaStream_t s) {
    count_launch();
    k_device_scales<<<1, 1, 0, s>>>(maxbits, n_rows, scales, err);
}
void launch_device_scales_exact(const unsigned long long* maxbits, unsigned long long n_rows,
                                const fbx::ScaleExc* exc, uint32_t n_exc, double* scales, unsigned long long* err,
                                cudaStream_t s) {
    count_launch();
    k_device_scales_exact<<<1, 1, 0, s>>>(maxbits, n_rows, exc, n_exc, scales, err);
}
void launch_quantizer_scales(const float* vals, uint64_t count, unsigned long long n_rows, const fbx::ScaleExc* exc,
                             uint32_t n_exc, double* out, cudaStream_t s) {
    if (count == 0) return;
    count_launch();
    const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 148ull * 8);
    k_quantizer_scales<<<(unsigned)blocks, 256, 0, s>>>(vals, count, n_rows, exc, n_exc, out);
}
void set_hist_smem_limit(int bytes) {
    cudaFuncSetAttribute(k_hist<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
void launch_hist(int width, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat, const uint32_t* rows,
                 const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                 const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                 unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s) {
    if (n_tiles == 0) return;
    dim3 grid(grid_x, n_tiles);
    count_launch();
    if (width == 2)
        k_hist<2><<<grid, kHistThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list, acc_prefix, st,
                                                   hist_acc, slot_pairs);
    else
        k_hist<1><<<grid, kHistThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list, acc_prefix, st,
                                                   hist_acc, slot_pairs);
}
void set_hist_lpf_smem_limit(int bytes) {
    cudaFuncSetAttribute(k_hist_lpf<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist_lpf<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
void launch_hist_lpf(int width, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat,
                     const uint32_t* rows, const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                     const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                     unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s) {
    if (n_tiles == 0) return;
    dim3 grid(grid_x, n_tiles);
    count_launch();
    if (width == 2)
        k_hist_lpf<2><<<grid, kHistLpfThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list, acc_prefix,
                                                          st, hist_acc, slot_pairs);
    else
        k_hist_lpf<1><<<grid, kHistLpfThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list, acc_prefix,
                                                          st, hist_acc, slot_pairs);
}
void set_hist_stage_smem_limit(int bytes) {
    cudaFuncSetAttribute(k_hist_stage<1, 2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist_stage<2, 2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist_stage<1, 4, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist_stage<2, 4, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
void set_hist_wide_smem_limit(int bytes) {
    cudaFuncSetAttribute(k_hist_stage<2, 2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(k_hist_stage<2, 4, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}
void launch_hist_wide(int stages, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat, const uint32_t* rows,
                      const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                      const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                      unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s) {
    if (n_tiles == 0) return;
    dim3 grid(grid_x, n_tiles);
    count_launch();
    if (stages == 4)
        k_hist_stage<2, 4, 8><<<grid, kHistLpfThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list,
                                                                  acc_prefix, st, hist_acc, slot_pairs);
    else
        k_hist_stage<2, 2, 8><<<grid, kHistLpfThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list,
                                                                  acc_prefix, st, hist_acc, slot_pairs);
}
void launch_hist_stage(int width, int stages, const TileDesc* tiles, uint32_t n_tiles, const TileFeat* tfeat,
                       const uint32_t* rows, const Pair* gpair, const NodeInfo* nodes, const uint32_t* acc_list,
                       const unsigned long long* acc_prefix, const TreeState* st, Pair* hist_acc,
                       unsigned long long slot_pairs, uint32_t grid_x, size_t smem, cudaStream_t s) {
    if (n_tiles == 0) return;
    dim3 grid(grid_x, n_tiles);
    count_launch();
#define FB_HS(W, S)                                                                                                \
    k_hist_stage<W, S, 32><<<grid, kHistLpfThreads, smem, s>>>(tiles, tfeat, rows, gpair, nodes, acc_list,         \
                                                              acc_prefix, st, hist_acc, slot_pairs)
    if (width == 2) {
        if (stages == 4) FB_HS(2, 4); else FB_HS(2, 2);
    } else {
        if (stages == 4) FB_HS(1, 4); else FB_HS(1, 2);
    }
#undef FB_HS
}
// The per-feature searches.  From kSplitWarpNodes nodes on: numeric features
// of up to kSplitWarpBins bins a warp each (k_split_num), the others a CTA
// each (k_split_feat).  Below (or without the lists) every feature of
// [feat_lo, feat_hi) a CTA: with few nodes, a warp's serial chain of 16 gain
// evaluations takes longer than a CTA's one per thread (measured on B200, C1:
// the warp form 15-18 us per level up to 16 nodes against 10-15, and 26 / 32
// against 32 / 55 us at 64 / 128 nodes).
constexpr uint32_t kSplitWarpNodes = 32;
static void launch_split_feats(const LevelArgs& a, uint32_t max_m, cudaStream_t s) {
    if (!a.split_cta || max_m < kSplitWarpNodes) {
        if (a.feat_hi > a.feat_lo) {
            LevelArgs all = a;
            all.split_cta = nullptr;
            count_launch();
            k_split_feat<<<dim3(max_m, a.feat_hi - a.feat_lo), kSplitThreads, 0, s>>>(all);
        }
        return;
    }
    if (a.n_split_num) {
        count_launch();
        k_split_num<<<dim3(max_m, (a.n_split_num + kSplitNumThreads / 32 - 1) / (kSplitNumThreads / 32)),
                      kSplitNumThreads, 0, s>>>(a);
    }
    if (a.n_split_cta) {
        count_launch();
        k_split_feat<<<dim3(max_m, a.n_split_cta), kSplitThreads, 0, s>>>(a);
    }
}
void launch_split(const LevelArgs& a, uint32_t max_m, cudaStream_t s) {
    launch_split_feats(a, max_m, s);
    count_launch();
    k_split_node<<<max_m, 32, 0, s>>>(a);
}
void launch_split_decide(const LevelArgs& a, uint32_t max_m, cudaStream_t s) {
    launch_split_feats(a, max_m, s);
    count_launch();
    k_split_node_decide<<<(max_m + 7) / 8, 256, 0, s>>>(a);
}
void launch_merge_decide(const LevelArgs& a, const SplitRec* all_best, const uint32_t* all_cats, uint32_t n_ranks,
                         uint32_t max_m, cudaStream_t s) {
    count_launch();
    k_merge_decide<<<(max_m + 255) / 256, 256, 0, s>>>(a, all_best, all_cats, n_ranks, max_m);
}
void launch_part_count(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s) {
    count_launch();
    k_part_count<<<max_chunks, kPartThreads, 0, s>>>(a);
}
void launch_part_scan(const LevelArgs& a, cudaStream_t s) { count_launch(); k_part_scan<<<1, 1024, 0, s>>>(a); }
void launch_part_scatter(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s) {
    count_launch();
    k_part_scatter<<<max_chunks, kPartThreads, 0, s>>>(a);
}
void launch_part_level(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s) {
    count_launch();
    k_part_level<<<max_chunks, kPartThreads, 0, s>>>(a);
}
void launch_tree_walk(const LevelArgs& a, uint32_t n_rows, cudaStream_t s, const GradArgs* next_grad, int gmode) {
    if (n_rows == 0) return;
    count_launch();
    // one resident wave: every CTA takes the same number of steps, so a grid
    // beyond what the SMs hold at once would run a second, nearly empty wave
    static const uint32_t wave8 =
        resident_grid(reinterpret_cast<const void*>(k_tree_walk<8, false>), kWalkThreads);
    static const uint32_t wave16 =
        resident_grid(reinterpret_cast<const void*>(k_tree_walk<16, false>), kWalkThreads);
    static const uint32_t wave8g = resident_grid(reinterpret_cast<const void*>(k_tree_walk<8, true>), kWalkThreads);
    static const uint32_t wave16g =
        resident_grid(reinterpret_cast<const void*>(k_tree_walk<16, true>), kWalkThreads);
    const bool narrow = a.walk_rec == nullptr || a.walk_stride <= 32;
    const uint32_t want = (n_rows + kWalkThreads - 1) / kWalkThreads;
    if (next_grad) {
        const uint32_t blocks = std::min<uint32_t>(want, narrow ? wave8g : wave16g);
        if (narrow) k_tree_walk<8, true><<<blocks, kWalkThreads, 0, s>>>(a, n_rows, *next_grad, gmode);
        else k_tree_walk<16, true><<<blocks, kWalkThreads, 0, s>>>(a, n_rows, *next_grad, gmode);
        return;
    }
    const GradArgs none{};
    const uint32_t blocks = std::min<uint32_t>(want, narrow ? wave8 : wave16);
    if (narrow) k_tree_walk<8, false><<<blocks, kWalkThreads, 0, s>>>(a, n_rows, none, 0);
    else k_tree_walk<16, false><<<blocks, kWalkThreads, 0, s>>>(a, n_rows, none, 0);
}
void launch_part_final(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s) {
    count_launch();
    k_part_final<<<max_chunks, kPartThreads, 0, s>>>(a);
}
void launch_leaf_final(const LevelArgs& a, uint32_t max_chunks, cudaStream_t s) {
    count_launch();
    k_leaf_final<<<max_chunks, kPartThreads, 0, s>>>(a);
}
void launch_tree_init(const LevelArgs& a, uint32_t n_local, uint32_t n_global, const unsigned long long* root_sum,
                      cudaStream_t s) {
    count_launch();
    k_tree_init<<<1, 32, 0, s>>>(a, n_local, n_global, root_sum);
}
__global__ void k_fill(float* p, uint64_t n, float v) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        p[i] = v;
}
void launch_fill(float* p, uint64_t n, float v, cudaStream_t s) {
    if (n == 0) return;
    count_launch();
    k_fill<<<(unsigned)std::min<uint64_t>((n + 255) / 256, 148ull * 16), 256, 0, s>>>(p, n, v);
}
void launch_iota(uint32_t* rows, uint32_t n, cudaStream_t s) {
    count_launch();
    k_iota<<<grad_grid(n), 256, 0, s>>>(rows, n);
}
void launch_records_to_columns(int width, const uint8_t* rec, uint32_t stride, uint64_t n_rows, uint32_t n_feats,
                               uint8_t* cols, cudaStream_t s) {
    const size_t smem = (size_t)kTrRows * (stride + 4);
    if (smem > 48 * 1024) {
        cudaFuncSetAttribute(k_records_to_columns<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(k_records_to_columns<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    const uint32_t grid = (uint32_t)std::min<uint64_t>((n_rows + kTrRows - 1) / kTrRows, 148ull * 8);
    count_launch();
    if (width == 2) k_records_to_columns<2><<<grid, 256, smem, s>>>(rec, stride, n_rows, n_feats, cols);
    else k_records_to_columns<1><<<grid, 256, smem, s>>>(rec, stride, n_rows, n_feats, cols);
}
void launch_transpose(int width, const uint8_t* src, uint8_t* dst, uint32_t n_rows, uint32_t n_feats,
                      uint32_t stride, uint64_t row0, cudaStream_t s) {
    count_launch();
    if (width == 2) k_transpose_block<2><<<148 * 16, 256, 0, s>>>(src, dst, n_rows, n_feats, stride, row0);
    else k_transpose_block<1><<<148 * 16, 256, 0, s>>>(src, dst, n_rows, n_feats, stride, row0);
}

// Explicit instantiations used by the host code.
template __global__ void k_hist<1>(const TileDesc*, const TileFeat*, const uint32_t*, const Pair*, const NodeInfo*,
                                   const uint32_t*, const unsigned long long*, const TreeState*, Pair*,
                                   unsigned long long);
template __global__ void k_hist<2>(const TileDesc*, const TileFeat*, const uint32_t*, const Pair*, const NodeInfo*,
                                   const uint32_t*, const unsigned long long*, const TreeState*, Pair*,
                                   unsigned long long);
template __global__ void k_hist_lpf<1>(const TileDesc*, const TileFeat*, const uint32_t*, const Pair*,
                                       const NodeInfo*, const uint32_t*, const unsigned long long*, const TreeState*,
                                       Pair*, unsigned long long);
template __global__ void k_hist_lpf<2>(const TileDesc*, const TileFeat*, const uint32_t*, const Pair*,
                                       const NodeInfo*, const uint32_t*, const unsigned long long*, const TreeState*,
                                       Pair*, unsigned long long);
template __global__ void k_transpose_block<1>(const uint8_t*, uint8_t*, uint32_t, uint32_t, uint32_t, uint64_t);
template __global__ void k_transpose_block<2>(const uint8_t*, uint8_t*, uint32_t, uint32_t, uint32_t, uint64_t);

}  // namespace fbg
