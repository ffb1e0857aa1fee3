// Tree prediction and QuadratureTreeSHAP kernels (sm_100a).
//
// Prediction restates Model::predict_margin_upto (model/tree.rs:498-510): one
// thread per row walks the trees in model order and adds each leaf value to
// the f32 margin.  SHAP restates the 8-point QuadratureTreeSHAP of
// model/explain.rs:198-400 with the same f32 operation order (explicit
// round-to-nearest intrinsics, no contraction), so each row's values equal the
// CPU engine's bit for bit.  The recursion is an explicit per-thread stack:
// QuadratureTreeSHAP visits every node of a tree whatever the row, so the
// threads of a warp walk the same nodes in the same order and only their
// feature values differ (no divergence on the traversal itself).
#include <cstdint>

#include "explain_kernels.cuh"

namespace fbg {

__constant__ float c_rule_nodes[kShapPoints];
__constant__ float c_rule_weights[kShapPoints];

__device__ __forceinline__ bool cat_goes_left(const uint32_t* words, uint32_t n_words, float v) {
    // data/categorical.rs:330-345 (XGBoost Decision)
    if (v < 0.0f || v >= 16777216.0f) return true;
    const uint32_t c = (uint32_t)v;
    if ((c >> 5) >= n_words) return true;
    return ((words[c >> 5] >> (c & 31)) & 1u) == 0u;
}

__device__ __forceinline__ bool node_goes_left(const DevNode& nd, const DevModel& m, uint32_t idx, float v) {
    const uint32_t flags = nd.meta >> 24;
    if (v != v) return (flags & kNodeDefaultLeft) != 0;  // tree.rs:84-96 goes_left
    if (flags & kNodeCategorical) return cat_goes_left(m.cat_words + m.cat_off[idx], m.cat_len[idx], v);
    return v < nd.val;
}

__global__ void k_predict(DevModel m, const float* __restrict__ X, uint64_t n, float base_margin,
                          float* __restrict__ out) {
    for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < n; r += (uint64_t)blockDim.x * gridDim.x) {
        const float* x = X + r * m.n_features;
        float acc = base_margin;
        for (uint32_t t = 0; t < m.n_trees; t++) {
            uint32_t i = m.tree_off[t];
            for (;;) {
                const DevNode nd = m.nodes[i];
                if ((nd.meta >> 24) & kNodeLeaf) { acc = __fadd_rn(acc, nd.val); break; }
                const uint32_t f = nd.meta & 0xffffffu;
                i = m.tree_off[t] + (uint32_t)(node_goes_left(nd, m, i, x[f]) ? nd.left : nd.right);
            }
        }
        out[r] = acc;
    }
}

// explain.rs:182-192
__device__ __forceinline__ float branch_weight(float cover, float parent) {
    if (parent <= 0.0f) return 0.5f;
    const float w = __fdiv_rn(cover, parent);
    return w < 1e-12f ? 1e-12f : w;
}

// explain.rs:198-216 extract_delta
__device__ __forceinline__ float extract_delta(const float* h, float pe, float px) {
    float acc = 0.0f;
    if (pe != 1.0f) {
        const float a = __fsub_rn(pe, 1.0f);
#pragma unroll
        for (int i = 0; i < kShapPoints; i++)
            acc = __fadd_rn(acc, __fdiv_rn(__fmul_rn(a, h[i]), __fadd_rn(1.0f, __fmul_rn(a, c_rule_nodes[i]))));
    }
    if (px != 1.0f) {
        const float a = __fsub_rn(px, 1.0f);
#pragma unroll
        for (int i = 0; i < kShapPoints; i++)
            acc = __fsub_rn(acc, __fdiv_rn(__fmul_rn(a, h[i]), __fadd_rn(1.0f, __fmul_rn(a, c_rule_nodes[i]))));
    }
    return acc;
}

constexpr float kUnseen = -999.0f;

struct Frame {
    float c[kShapPoints];   // input coefficients of this node
    float hl[kShapPoints];  // left child's result
    float wp;
    float p_old;
    float pe;
    uint32_t idx;
    uint32_t stage;
};

// One thread per row; `path` and `tc` are this thread's per-feature scratch
// (feature f of thread t at [f * T + t]).
__global__ void __launch_bounds__(128) k_shap(DevModel m, const float* __restrict__ X, uint64_t n,
                                              float bias, float root_mean, float* __restrict__ out,
                                              float* __restrict__ path, float* __restrict__ tc) {
    const uint32_t F = m.n_features;
    const uint64_t T = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    Frame st[kMaxShapDepth + 1];
    for (uint64_t r = tid; r < n; r += T) {
        const float* x = X + r * F;
        float* p = out + r * (F + 1);
        for (uint32_t f = 0; f <= F; f++) p[f] = 0.0f;
        for (uint32_t f = 0; f < F; f++) path[f * T + tid] = kUnseen;
        for (uint32_t t = 0; t < m.n_trees; t++) {
            const DevNode* nodes = m.nodes + m.tree_off[t];
            const uint32_t gbase = m.tree_off[t];
            if ((nodes[0].meta >> 24) & kNodeLeaf) continue;  // explain.rs:393-400 run
            for (uint32_t f = 0; f < F; f++) tc[f * T + tid] = 0.0f;
            int sp = 0;
#pragma unroll
            for (int i = 0; i < kShapPoints; i++) st[0].c[i] = 1.0f;
            st[0].wp = 1.0f;
            st[0].idx = 0;
            st[0].stage = 0;
            float h[kShapPoints];
            bool have_ret = false;  // h holds a child's result for the top frame
            while (sp >= 0) {
                Frame& fr = st[sp];
                const DevNode nd = nodes[fr.idx];
                const uint32_t feat = nd.meta & 0xffffffu;
                if (have_ret) {
                    // return from visit_child(stage): explain.rs:345-349
                    const float px = fr.p_old == kUnseen ? 1.0f : fr.p_old;
                    tc[feat * T + tid] = __fadd_rn(tc[feat * T + tid], extract_delta(h, fr.pe, px));
                    path[feat * T + tid] = fr.p_old;
                    if (fr.stage == 0) {
#pragma unroll
                        for (int i = 0; i < kShapPoints; i++) fr.hl[i] = h[i];
                        fr.stage = 1;
                        have_ret = false;
                    } else {
#pragma unroll
                        for (int i = 0; i < kShapPoints; i++) h[i] = __fadd_rn(fr.hl[i], h[i]);
                        sp--;
                        continue;  // have_ret stays true for the parent frame
                    }
                }
                // visit_child(stage): explain.rs:312-350
                const bool left_side = fr.stage == 0;
                const int32_t child = left_side ? nd.left : nd.right;
                const float cw = branch_weight(nodes[child].hess, nd.hess);
                const bool gl = node_goes_left(nd, m, gbase + fr.idx, x[feat]);
                const bool sat = left_side ? gl : !gl;
                const float p_old = path[feat * T + tid];
                const float pe = sat ? __fdiv_rn(p_old == kUnseen ? 1.0f : p_old, cw) : 0.0f;
                float cc[kShapPoints];
                const float ae = __fsub_rn(pe, 1.0f);
#pragma unroll
                for (int i = 0; i < kShapPoints; i++)
                    cc[i] = __fmul_rn(fr.c[i], __fadd_rn(1.0f, __fmul_rn(ae, c_rule_nodes[i])));
                if (p_old != kUnseen) {
                    const float ao = __fsub_rn(p_old, 1.0f);
                    if (ao != 0.0f) {
#pragma unroll
                        for (int i = 0; i < kShapPoints; i++)
                            cc[i] = __fdiv_rn(cc[i], __fadd_rn(1.0f, __fmul_rn(ao, c_rule_nodes[i])));
                    }
                }
                path[feat * T + tid] = pe;
                fr.p_old = p_old;
                fr.pe = pe;
                const float wpc = __fmul_rn(fr.wp, cw);
                const DevNode ch = nodes[child];
                if ((ch.meta >> 24) & kNodeLeaf) {
                    // run_node on a leaf: explain.rs:353-358
                    const float ls = __fmul_rn(wpc, ch.val);
#pragma unroll
                    for (int i = 0; i < kShapPoints; i++) h[i] = __fmul_rn(__fmul_rn(cc[i], ls), c_rule_weights[i]);
                    have_ret = true;
                } else {
                    Frame& nf = st[++sp];
#pragma unroll
                    for (int i = 0; i < kShapPoints; i++) nf.c[i] = cc[i];
                    nf.wp = wpc;
                    nf.idx = (uint32_t)child;
                    nf.stage = 0;
                }
            }
            for (uint32_t f = 0; f < F; f++) p[f] = __fadd_rn(p[f], tc[f * T + tid]);
        }
        p[F] = __fadd_rn(p[F], root_mean);  // explain.rs:725-726
        p[F] = __fadd_rn(p[F], bias);
    }
}

// explain.rs:690-701 leaf_row: the node index each tree's traversal ends
// at, as f32, n x n_trees.
__global__ void k_pred_leaf(DevModel m, const float* __restrict__ X, uint64_t n, float* __restrict__ out) {
    for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < n; r += (uint64_t)blockDim.x * gridDim.x) {
        const float* x = X + r * m.n_features;
        for (uint32_t t = 0; t < m.n_trees; t++) {
            const uint32_t base = m.tree_off[t];
            uint32_t i = 0;
            for (;;) {
                const DevNode nd = m.nodes[base + i];
                if ((nd.meta >> 24) & kNodeLeaf) break;
                const uint32_t f = nd.meta & 0xffffffu;
                i = (uint32_t)(node_goes_left(nd, m, base + i, x[f]) ? nd.left : nd.right);
            }
            out[r * m.n_trees + t] = (float)i;
        }
    }
}

// explain.rs:729-760 saabas_row (approx_contribs): along each tree's path,
// the change of the cover-weighted node mean goes to the split feature.
// `means` are the per-node f32 means of explain.rs:409-421, in node order.
// Per tree the deltas gather in tc (one feature may split several times on
// a path), then add to the row's totals, as the reference does; shared
// memory holds tc and the totals as [feature][thread].
constexpr int kApproxThreads = 128;
__global__ void __launch_bounds__(kApproxThreads) k_pred_approx(DevModel m, const float* __restrict__ means,
                                                                const float* __restrict__ X, uint64_t n, float bias,
                                                                float* __restrict__ out) {
    extern __shared__ float sm_approx[];
    const uint32_t F = m.n_features, nc = F + 1, t = threadIdx.x;
    float* p = sm_approx;                       // [nc][kApproxThreads]
    float* tc = sm_approx + nc * kApproxThreads;  // [nc][kApproxThreads]
    for (uint64_t r0 = (uint64_t)blockIdx.x * kApproxThreads; r0 < n; r0 += (uint64_t)gridDim.x * kApproxThreads) {
        const uint64_t r = r0 + t;
        if (r < n) {
            const float* x = X + r * F;
            for (uint32_t c = 0; c < nc; c++) { p[c * kApproxThreads + t] = 0.0f; tc[c * kApproxThreads + t] = 0.0f; }
            for (uint32_t tr = 0; tr < m.n_trees; tr++) {
                const uint32_t base = m.tree_off[tr];
                float node_value = means[base];
                float& tb = tc[F * kApproxThreads + t];
                tb = __fadd_rn(tb, node_value);
                uint32_t touched[kMaxShapDepth + 1];
                uint32_t nt = 0;
                DevNode nd = m.nodes[base];
                if (!((nd.meta >> 24) & kNodeLeaf)) {
                    uint32_t i = 0, split = 0;
                    while (!((nd.meta >> 24) & kNodeLeaf)) {
                        split = nd.meta & 0xffffffu;
                        i = (uint32_t)(node_goes_left(nd, m, base + i, x[split]) ? nd.left : nd.right);
                        const float nv = means[base + i];
                        float& ts = tc[split * kApproxThreads + t];
                        ts = __fadd_rn(ts, __fsub_rn(nv, node_value));
                        if (nt <= (uint32_t)kMaxShapDepth) touched[nt++] = split;
                        node_value = nv;
                        nd = m.nodes[base + i];
                    }
                    float& ts = tc[split * kApproxThreads + t];
                    ts = __fadd_rn(ts, __fsub_rn(nd.val, node_value));
                }
                // p[c] += tc[c] for every column; untouched columns hold 0
                for (uint32_t k = 0; k < nt; k++) {
                    const uint32_t f = touched[k];
                    float& tf = tc[f * kApproxThreads + t];
                    p[f * kApproxThreads + t] = __fadd_rn(p[f * kApproxThreads + t], tf);
                    tf = 0.0f;
                }
                p[F * kApproxThreads + t] = __fadd_rn(p[F * kApproxThreads + t], tb);
                tb = 0.0f;
            }
            float* o = out + r * nc;
            for (uint32_t c = 0; c < F; c++) o[c] = p[c * kApproxThreads + t];
            o[F] = __fadd_rn(p[F * kApproxThreads + t], bias);
        }
    }
}

void launch_pred_leaf(const DevModel& m, const float* X, uint64_t n, float* out, cudaStream_t s) {
    if (n == 0) return;
    uint64_t blocks = (n + 255) / 256;
    if (blocks > 148ull * 64) blocks = 148ull * 64;
    count_launch();
    k_pred_leaf<<<(unsigned)blocks, 256, 0, s>>>(m, X, n, out);
}

// The same for models with more features than shared memory holds per row:
// the row's totals accumulate in its output row (global memory, the same f32
// additions in the same order) and a tree's deltas in a few per-thread slots,
// one per feature on the path, visited in the order the shared-memory kernel
// visits its columns.
__global__ void __launch_bounds__(kApproxThreads) k_pred_approx_wide(DevModel m, const float* __restrict__ means,
                                                                     const float* __restrict__ X, uint64_t n,
                                                                     float bias, float* __restrict__ out) {
    const uint32_t F = m.n_features, nc = F + 1;
    for (uint64_t r = (uint64_t)blockIdx.x * kApproxThreads + threadIdx.x; r < n;
         r += (uint64_t)gridDim.x * kApproxThreads) {
        const float* x = X + r * F;
        float* o = out + r * nc;
        for (uint32_t c = 0; c < F; c++) o[c] = 0.0f;
        float pb = 0.0f;  // bias column total
        for (uint32_t tr = 0; tr < m.n_trees; tr++) {
            const uint32_t base = m.tree_off[tr];
            float node_value = means[base];
            const float tb = __fadd_rn(0.0f, node_value);
            uint32_t touched[kMaxShapDepth + 1];
            uint32_t slot_feat[kMaxShapDepth + 1];
            float slot_val[kMaxShapDepth + 1];
            uint32_t nt = 0, ns = 0;
            auto slot_of = [&](uint32_t f) {
                for (uint32_t q = 0; q < ns; q++)
                    if (slot_feat[q] == f) return q;
                slot_feat[ns] = f;
                slot_val[ns] = 0.0f;
                return ns++;
            };
            DevNode nd = m.nodes[base];
            if (!((nd.meta >> 24) & kNodeLeaf)) {
                uint32_t i = 0, split = 0, q = 0;
                while (!((nd.meta >> 24) & kNodeLeaf)) {
                    split = nd.meta & 0xffffffu;
                    i = (uint32_t)(node_goes_left(nd, m, base + i, x[split]) ? nd.left : nd.right);
                    const float nv = means[base + i];
                    if (nt > (uint32_t)kMaxShapDepth) break;  // trees are at most kMaxShapDepth deep
                    q = slot_of(split);
                    slot_val[q] = __fadd_rn(slot_val[q], __fsub_rn(nv, node_value));
                    touched[nt++] = split;
                    node_value = nv;
                    nd = m.nodes[base + i];
                }
                slot_val[q] = __fadd_rn(slot_val[q], __fsub_rn(nd.val, node_value));
            }
            for (uint32_t k = 0; k < nt; k++) {
                const uint32_t q = slot_of(touched[k]);
                o[touched[k]] = __fadd_rn(o[touched[k]], slot_val[q]);
                slot_val[q] = 0.0f;
            }
            pb = __fadd_rn(pb, tb);
        }
        o[F] = __fadd_rn(pb, bias);
    }
}

void launch_pred_approx(const DevModel& m, const float* means, const float* X, uint64_t n, float bias, float* out,
                        cudaStream_t s) {
    if (n == 0) return;
    const size_t smem = 2ull * (m.n_features + 1) * kApproxThreads * sizeof(float);
    if (smem > 227 * 1024) {
        uint64_t blocks = (n + kApproxThreads - 1) / kApproxThreads;
        if (blocks > 148ull * 16) blocks = 148ull * 16;
        count_launch();
        k_pred_approx_wide<<<(unsigned)blocks, kApproxThreads, 0, s>>>(m, means, X, n, bias, out);
        return;
    }
    cudaFuncSetAttribute(k_pred_approx, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    uint64_t blocks = (n + kApproxThreads - 1) / kApproxThreads;
    if (blocks > 148ull * 16) blocks = 148ull * 16;
    count_launch();
    k_pred_approx<<<(unsigned)blocks, kApproxThreads, smem, s>>>(m, means, X, n, bias, out);
}

size_t approx_smem_bytes(uint32_t n_features) { return 2ull * (n_features + 1) * kApproxThreads * sizeof(float); }

void upload_shap_rule(const float* nodes, const float* weights, cudaStream_t s) {
    cudaMemcpyToSymbolAsync(c_rule_nodes, nodes, sizeof(float) * kShapPoints, 0, cudaMemcpyHostToDevice, s);
    cudaMemcpyToSymbolAsync(c_rule_weights, weights, sizeof(float) * kShapPoints, 0, cudaMemcpyHostToDevice, s);
}

void launch_predict(const DevModel& m, const float* X, uint64_t n, float base_margin, float* out, cudaStream_t s) {
    if (n == 0) return;
    uint64_t blocks = (n + 255) / 256;
    if (blocks > 148ull * 64) blocks = 148ull * 64;
    count_launch();
    k_predict<<<(unsigned)blocks, 256, 0, s>>>(m, X, n, base_margin, out);
}

// At most one wave of 128-thread CTAs: the kernel's 54 registers per thread
// allow 9 per SM, and a second partial wave would leave a tail.
uint64_t shap_threads(uint64_t n) {
    uint64_t t = ((n + 127) / 128) * 128;
    const uint64_t cap = 148ull * 9 * 128;
    return t < cap ? t : cap;
}

void launch_shap(const DevModel& m, const float* X, uint64_t n, float bias, float root_mean, float* out,
                 float* path, float* tc, cudaStream_t s) {
    if (n == 0) return;
    const uint64_t T = shap_threads(n);
    count_launch();
    k_shap<<<(unsigned)(T / 128), 128, 0, s>>>(m, X, n, bias, root_mean, out, path, tc);
}

}  // namespace fbg
