// Device model layout shared by the prediction and SHAP kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace fbg {

// Counts this library's kernel launches (fbgpu_launch_count).
void count_launch();

constexpr int kShapPoints = 8;     // explain.rs:32 POINTS
constexpr int kMaxShapDepth = 14;  // types.rs:424 MAX_DEPTH_LIMIT

constexpr uint32_t kNodeLeaf = 1u;
constexpr uint32_t kNodeDefaultLeft = 2u;
constexpr uint32_t kNodeCategorical = 4u;

// One tree node in 16 bytes: val is the leaf value of a leaf or the split
// condition of a numeric split; children are tree-local indices; meta holds
// the feature (low 24 bits) and the flags (high 8 bits).
struct DevNode {
    float val;
    int32_t left;
    int32_t right;
    uint32_t meta;
    float hess;
    uint32_t pad[3];
};
static_assert(sizeof(DevNode) == 32, "DevNode layout");

struct DevModel {
    const DevNode* nodes;       // all trees back to back
    const uint32_t* tree_off;   // n_trees + 1
    const uint32_t* cat_off;    // per node: first word in cat_words
    const uint32_t* cat_len;    // per node: words of its category set
    const uint32_t* cat_words;
    uint32_t n_trees;
    uint32_t n_features;
};

void upload_shap_rule(const float* nodes, const float* weights, cudaStream_t s);
void launch_pred_leaf(const DevModel& m, const float* X, uint64_t n, float* out, cudaStream_t s);
void launch_pred_approx(const DevModel& m, const float* means, const float* X, uint64_t n, float bias, float* out,
                        cudaStream_t s);
size_t approx_smem_bytes(uint32_t n_features);
void launch_predict(const DevModel& m, const float* X, uint64_t n, float base_margin, float* out, cudaStream_t s);
uint64_t shap_threads(uint64_t n);
void launch_shap(const DevModel& m, const float* X, uint64_t n, float bias, float root_mean, float* out,
                 float* path, float* tc, cudaStream_t s);

}  // namespace fbg
