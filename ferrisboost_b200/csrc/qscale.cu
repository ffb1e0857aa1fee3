// C entry points for the quantizer scales (qscale.h): the scales of given
// bounds on the host or the device, and a digest of the scales of a range of
// f32 bit patterns.  Training computes its scales with the same functions
// (k_device_scales_exact); these let the tests check them against the
// reference's pow2_scale on every positive f32.
#include <omp.h>

#include <cuda_runtime.h>

#include "ctx.h"

namespace fbg {
namespace {

uint64_t digest_mix(uint32_t bits, double scale) {
    uint64_t s;
    std::memcpy(&s, &scale, 8);
    uint64_t z = s ^ ((uint64_t)bits * 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <class F> fbgpu_status guarded(F&& f) {
    try {
        f();
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

}  // namespace
}  // namespace fbg

extern "C" fbgpu_status fbgpu_quantizer_scales(int32_t device, const float* max_abs, uint64_t count, uint64_t n_rows,
                                               double* out) {
    using namespace fbg;
    return guarded([&] {
        if (count && (!max_abs || !out)) throw InputError("max_abs and out must not be null");
        const std::vector<fbx::ScaleExc> exc = build_scale_exceptions(n_rows);
        if (device < 0) {
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)count; i++)
                out[i] = fbx::scale_of_exp(fbx::scale_exp_exact((double)max_abs[i], n_rows, exc.data(),
                                                                (uint32_t)exc.size()));
            return;
        }
        FB_CUDA_CHECK(cudaSetDevice(device));
        cudaStream_t s = nullptr;
        FB_CUDA_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        struct Owner {
            cudaStream_t s;
            ~Owner() { cudaStreamDestroy(s); }
        } owner{s};
        DevMem dv, dout, dexc;
        dv.alloc(std::max<uint64_t>(count, 1) * 4);
        dout.alloc(std::max<uint64_t>(count, 1) * 8);
        dexc.alloc(sizeof(fbx::ScaleExc) * std::max<size_t>(exc.size(), 1));
        if (count) FB_CUDA_CHECK(cudaMemcpyAsync(dv.p, max_abs, count * 4, cudaMemcpyHostToDevice, s));
        if (!exc.empty())
            FB_CUDA_CHECK(cudaMemcpyAsync(dexc.p, exc.data(), sizeof(fbx::ScaleExc) * exc.size(),
                                          cudaMemcpyHostToDevice, s));
        launch_quantizer_scales(dv.as<float>(), count, n_rows, dexc.as<fbx::ScaleExc>(), (uint32_t)exc.size(),
                                dout.as<double>(), s);
        FB_CUDA_CHECK(cudaGetLastError());
        if (count) FB_CUDA_CHECK(cudaMemcpyAsync(out, dout.p, count * 8, cudaMemcpyDeviceToHost, s));
        FB_CUDA_CHECK(cudaStreamSynchronize(s));
    });
}

extern "C" uint64_t fbgpu_quantizer_scale_digest(uint32_t lo_bits, uint32_t hi_bits, uint64_t n_rows) {
    using namespace fbg;
    const std::vector<fbx::ScaleExc> exc = build_scale_exceptions(n_rows);
    uint64_t sum = 0;
#pragma omp parallel for schedule(static) reduction(+ : sum)
    for (int64_t b = (int64_t)lo_bits; b < (int64_t)hi_bits; b++) {
        float f;
        const uint32_t u = (uint32_t)b;
        std::memcpy(&f, &u, 4);
        sum += digest_mix(u, fbx::scale_of_exp(fbx::scale_exp_exact((double)f, n_rows, exc.data(),
                                                                     (uint32_t)exc.size())));
    }
    return sum;
}
