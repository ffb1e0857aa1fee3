// Throughput ceiling of the exact histogram update, measured alone.
//
// k_hist_stage (train_kernels.cu) adds each (row, feature) gradient pair to
// a shared-memory histogram as two 64-bit sums modulo 2^64, each kept as two
// 32-bit planes.  These kernels run the same update schemes with the rows
// generated in registers (no global loads, no staging), every lane adding to
// its own column of a [bin][plane][32 lanes] histogram of 256 bins shared by
// the CTA's 32 warps, so their rate is what the shared-memory atomics alone
// allow.  fbgpu_hist_atomic_ceiling times one scheme with CUDA events.
//
//   0  the low word by a returning 32-bit atomic, its carry into the high
//      word's atomic (add.cc / addc), g then h: 4 atomics per update
//   1  the same four atomics, issued for 4 updates at a time: the 8
//      returning low-word atomics first, then the 8 high-word ones
//   2  one native 64-bit shared atomic per sum (2 per update)
//   3  four non-returning 32-bit atomics per update (no carry: not exact;
//      the pipe's own ceiling for four shared atomics)
#include <cuda_runtime.h>

#include "ctx.h"

namespace fbg {
namespace {

constexpr uint32_t kCeilThreads = 1024;
constexpr uint32_t kCeilBins = 256;

__device__ __forceinline__ uint32_t xs32(uint32_t& s) {
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    return s;
}

__device__ __forceinline__ uint32_t carry_hi(uint32_t old, uint32_t vl, uint32_t vh) {
    uint32_t sum, hi_add;
    asm("add.cc.u32 %0, %2, %3;\n\taddc.u32 %1, %4, 0;" : "=r"(sum), "=r"(hi_add) : "r"(old), "r"(vl), "r"(vh));
    (void)sum;
    return hi_add;
}

template <int SCHEME>
__global__ void __launch_bounds__(kCeilThreads) k_hist_ceiling(uint32_t iters, unsigned long long* sink) {
    extern __shared__ uint32_t sm[];
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t j = threadIdx.x; j < kCeilBins * 128u; j += blockDim.x) sm[j] = 0u;
    __syncthreads();
    uint32_t s = 0x9E3779B9u ^ (blockIdx.x * 7919u + threadIdx.x * 104729u);
    uint32_t* col = sm + lane;
    for (uint32_t it = 0; it < iters; it += 4) {
        uint32_t bin[4], gl[4], gh[4], hl[4], hh[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint32_t r = xs32(s);
            bin[q] = r & (kCeilBins - 1);
            gl[q] = r * 2654435761u;
            gh[q] = (r >> 24) - 128u;  // a signed value of about 40 bits
            hl[q] = r ^ 0x5bd1e995u;
            hh[q] = r >> 26;
        }
        if (SCHEME == 0) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t* w = col + bin[q] * 128u;
                atomicAdd(w + 32, carry_hi(atomicAdd(w, gl[q]), gl[q], gh[q]));
                atomicAdd(w + 96, carry_hi(atomicAdd(w + 64, hl[q]), hl[q], hh[q]));
            }
        } else if (SCHEME == 1) {
            uint32_t og[4], oh[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t* w = col + bin[q] * 128u;
                og[q] = atomicAdd(w, gl[q]);
                oh[q] = atomicAdd(w + 64, hl[q]);
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t* w = col + bin[q] * 128u;
                atomicAdd(w + 32, carry_hi(og[q], gl[q], gh[q]));
                atomicAdd(w + 96, carry_hi(oh[q], hl[q], hh[q]));
            }
        } else if (SCHEME == 2) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                // 64-bit words: [bin][g, h][32 lanes] over the same 128 KiB
                unsigned long long* w = reinterpret_cast<unsigned long long*>(sm) + bin[q] * 64u + lane;
                atomicAdd(w, ((unsigned long long)gh[q] << 32) | gl[q]);
                atomicAdd(w + 32, ((unsigned long long)hh[q] << 32) | hl[q]);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint32_t* w = col + bin[q] * 128u;
                atomicAdd(w, gl[q]);
                atomicAdd(w + 32, gh[q]);
                atomicAdd(w + 64, hl[q]);
                atomicAdd(w + 96, hh[q]);
            }
        }
    }
    __syncthreads();
    unsigned long long acc = 0;
    for (uint32_t j = threadIdx.x; j < kCeilBins * 128u; j += blockDim.x) acc += sm[j];
    atomicAdd(sink, acc);
}

template <int SCHEME>
float time_scheme(uint32_t iters, int sms, unsigned long long* sink) {
    const size_t smem = kCeilBins * 128u * 4u;
    FB_CUDA_CHECK(cudaFuncSetAttribute(k_hist_ceiling<SCHEME>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaEvent_t e0, e1;
    FB_CUDA_CHECK(cudaEventCreate(&e0));
    FB_CUDA_CHECK(cudaEventCreate(&e1));
    count_launch();
    k_hist_ceiling<SCHEME><<<sms, kCeilThreads, smem>>>(iters / 8, sink);  // warm-up
    FB_CUDA_CHECK(cudaEventRecord(e0));
    count_launch();
    k_hist_ceiling<SCHEME><<<sms, kCeilThreads, smem>>>(iters, sink);
    FB_CUDA_CHECK(cudaEventRecord(e1));
    FB_CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.0f;
    FB_CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return ms;
}

}  // namespace
}  // namespace fbg

extern "C" fbgpu_status fbgpu_hist_atomic_ceiling(int32_t device, int32_t scheme, uint32_t iters,
                                                  double* updates_per_s) {
    using namespace fbg;
    try {
        if (scheme < 0 || scheme > 3) throw InputError("scheme must be 0..3");
        if (iters < 8 || iters % 8) throw InputError("iters must be a positive multiple of 8");
        if (!updates_per_s) throw InputError("updates_per_s is null");
        FB_CUDA_CHECK(cudaSetDevice(device));
        int sms = 148;
        FB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        DevMem sink;
        sink.alloc(8);
        FB_CUDA_CHECK(cudaMemset(sink.p, 0, 8));
        unsigned long long* sk = sink.as<unsigned long long>();
        float ms = scheme == 0 ? time_scheme<0>(iters, sms, sk)
                 : scheme == 1 ? time_scheme<1>(iters, sms, sk)
                 : scheme == 2 ? time_scheme<2>(iters, sms, sk)
                               : time_scheme<3>(iters, sms, sk);
        *updates_per_s = (double)sms * kCeilThreads * iters / (ms / 1000.0);
        return FBGPU_OK;
    } catch (const InputError& ex) {
        noalloc_set_error(ex.what());
        return FBGPU_EINPUT;
    } catch (const CudaError& ex) {
        noalloc_set_error(ex.what());
        return FBGPU_ECUDA;
    } catch (const std::exception& ex) {
        noalloc_set_error(ex.what());
        return FBGPU_EINTERNAL;
    }
}
