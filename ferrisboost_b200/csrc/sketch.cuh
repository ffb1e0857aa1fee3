// Dataset preparation on the device: the weighted quantile sketch of
// src/data/sketch.rs (unit weights) and dense quantization into the row
// records the training context reads (src/source/dense.rs:288-308).
//
// The sketch is a restatement, not an approximation of it: every chunk
// summary, merge, compression and cut selection performs the same f32
// operations as the sequential reference, so the cuts are bit-identical to
// the host engine's (and the CPU oracle's) for the same input.
#pragma once
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace fbg {

// Largest sketch summary the device path supports: max_bin <= 1024
// (limit = max_bin x 16 entries, sketch.rs:73), which also bounds the bins
// the device split search accepts.
constexpr uint32_t kSketchMaxLimit = 16384;

// A dense f32 matrix in one contiguous buffer: element (r, f) at
// p[r * rs + f * cs] (row-major: rs = F, cs = 1; column-major, one column
// per feature back to back: rs = 1, cs = n).
struct HostMatrix {
    const float* p;
    uint64_t rs, cs;
    float at(uint64_t r, uint32_t f) const { return p[r * rs + (uint64_t)f * cs]; }
};

// An f32 matrix (n x F) resident on one device in the layout of its host
// source, with the sketch and binning passes over it.  All work runs on
// `stream` of the current device.
class DeviceMatrix {
   public:
    // threads: host threads copying into the pinned staging (0: the OpenMP default)
    DeviceMatrix(const HostMatrix& X_host, uint64_t n, uint32_t F, cudaStream_t stream, int threads = 0);
    ~DeviceMatrix();
    DeviceMatrix(const DeviceMatrix&) = delete;
    DeviceMatrix& operator=(const DeviceMatrix&) = delete;

    // sketch.rs:128-302 cuts of the listed numeric features with unit
    // weights (FeatureSketch::push of every non-NaN value in row order, then
    // cuts(max_bin)).  per[i] receives the cuts of feats[i].
    void numeric_cuts(uint32_t max_bin, const std::vector<uint32_t>& feats, std::vector<std::vector<float>>& per);
    // categorical.rs scan of the listed features: the largest valid code
    // (-1 when none), and the first feature (in list order) holding a value
    // that is not a category code (-1 when none).
    void categorical_scan(const std::vector<uint32_t>& feats, std::vector<int32_t>& max_code, int64_t& bad_feat);
    // dense.rs:288-308 quantize_dense into one row-record block: record r of
    // `dst` (stride bytes, zero padded) holds the bins of feats[0..n_feats)
    // at byte i x width.  Cuts are the dataset's flat cuts and F+1 offsets
    // (device copies); NaN -> the missing sentinel (255 / 65535), categorical
    // codes -> their bin.  Returns true if any value of these features is
    // +-inf or f32::MAX (reserved: dense.rs:300, python/mod.rs:4063 reject_inf).
    bool bin_block(const uint32_t* feats, uint32_t n_feats, uint32_t width, const float* d_cuts,
                   const uint32_t* d_offsets, const uint8_t* d_cat, uint8_t* dst, uint32_t stride);
    // Features holding at least one NaN (1) or none (0), F entries.
    std::vector<uint8_t> nan_features();

   private:
    uint64_t n_;
    uint32_t F_;
    uint64_t rs_, cs_;  // element (r, f) at x_[r * rs_ + f * cs_]
    cudaStream_t s_;
    float* x_ = nullptr;
    size_t x_cap_ = 0;  // the block's size (dev_alloc)
};

}  // namespace fbg
