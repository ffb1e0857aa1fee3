// Power-of-two quantizer scales, identical on the host and the device.
//
// The reference quantizes each round's gradients with
//   scale = 2^clamp(floor(log2(raw)), -1000, 1000),  raw = (2^62 / n_rows) / max_abs
// (types.rs:366-385 pow2_scale), where log2 is the host C library's.  For a
// positive finite raw, floor(log2(raw)) is the binary exponent of raw
// (ilogb) except where log2 rounds up to the next integer, which a
// faithfully rounded log2 can do only when raw lies within about one unit in
// the last place of the result below a power of two.  max_abs here is always
// an f32 value (the largest |g| or |h| over f32 gradients, widened exactly),
// and f32 values are far coarser than that window, so for each power of two
// at most a few f32 values come near it.  The host lists, for a run's row
// count, every f32 max_abs around each power of two where its own
// floor(log2) and the binary exponent differ, with its own answer
// (build_scale_exceptions); both sides then take the binary exponent unless
// the list holds max_abs.  Every positive f32 is checked against the
// reference restatement by a digest over the whole range
// (tests/test_scales.py).
#pragma once
#include <cstdint>
#include <cmath>

#include "fexp.h"

namespace fbx {

// A max_abs (the bits of its f64 value) whose exponent is not raw's binary
// exponent, and the exponent to use.
struct ScaleExc {
    uint64_t bits;
    int32_t k;
    int32_t pad;
};
constexpr int32_t kScaleOne = INT32_MIN;  // the reference returns 1.0 (no positive finite raw)

FB_HD double scale_budget(uint64_t n_rows) {
    const uint64_t n = n_rows ? n_rows : 1;
#ifdef __CUDA_ARCH__
    return __ddiv_rn(4611686018427387904.0, __ull2double_rn(n));
#else
    return 4611686018427387904.0 / (double)n;
#endif
}

// The clamped binary exponent of raw, or kScaleOne.
FB_HD int32_t scale_exp_ilogb(double max_abs, uint64_t n_rows) {
#ifdef __CUDA_ARCH__
    if (!(max_abs > 0.0) || !isfinite(max_abs)) return kScaleOne;
    const double raw = __ddiv_rn(scale_budget(n_rows), max_abs);
    if (!isfinite(raw) || raw <= 0.0) return kScaleOne;
    int k = ilogb(raw);
#else
    if (!(max_abs > 0.0) || !std::isfinite(max_abs)) return kScaleOne;
    const double raw = scale_budget(n_rows) / max_abs;
    if (!std::isfinite(raw) || raw <= 0.0) return kScaleOne;
    int k = std::ilogb(raw);
#endif
    return k < -1000 ? -1000 : (k > 1000 ? 1000 : k);
}

// The reference's exponent: the binary exponent unless the exception list
// (sorted by bits) holds max_abs.
FB_HD int32_t scale_exp_exact(double max_abs, uint64_t n_rows, const ScaleExc* exc, uint32_t n_exc) {
    const int32_t k = scale_exp_ilogb(max_abs, n_rows);
    if (k == kScaleOne) return k;
    uint64_t bits;
#ifdef __CUDA_ARCH__
    bits = (uint64_t)__double_as_longlong(max_abs);
#else
    std::memcpy(&bits, &max_abs, 8);
#endif
    uint32_t lo = 0, hi = n_exc;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) / 2;
        if (exc[mid].bits < bits) lo = mid + 1;
        else hi = mid;
    }
    return lo < n_exc && exc[lo].bits == bits ? exc[lo].k : k;
}

FB_HD double scale_of_exp(int32_t k) { return k == kScaleOne ? 1.0 : pow2i(k); }

}  // namespace fbx
