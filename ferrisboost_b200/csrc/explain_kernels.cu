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
#include <cstdlib>

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

// ---------------------------------------------------------------------------
// QuadratureTreeSHAP with one lane per quadrature point.  A warp explains four
// rows at a time: lane 8g + i holds point i of row g.  The traversal is the
// same DFS as k_shap, identical for every row, so all 32 lanes stay in step.
// The per-edge factors that do not depend on the row are precomputed per
// tree (ShapEdges: the branch weight cw, 1/cw, and for each point the factor
// 1 + (1/cw - 1) x_i and its reciprocal; the not-satisfied factor 1 - x_i is a
// constant), so a visit is a few multiplies per lane instead of up to 25 f32
// divisions per row.  Dividing by a factor becomes multiplying by its
// reciprocal and the 8-point sums are reduced by butterfly shuffles, so the
// results differ from the reference in the last bits (the contract's bar is
// 1e-5 absolute; explain.rs:198-216, 312-358 give the recurrence).  The path
// probability of a feature is read from the DFS frames themselves: the
// deepest ancestor frame that splits on the same feature.
__constant__ float c_f0[kShapPoints];  // 1 - x_i (not satisfied: p_e = 0)
__constant__ float c_r0[kShapPoints];  // 1 / (1 - x_i)

constexpr int kShapQWarps = 4;
constexpr int kShapQFrames = kMaxShapDepth + 1;

__global__ void __launch_bounds__(32 * kShapQWarps) k_shap_q(DevModel m, ShapEdges e, const float* __restrict__ X,
                                                            uint64_t n, float bias, float root_mean,
                                                            float* __restrict__ out, uint32_t phi_in_smem) {
    extern __shared__ float sphi[];                       // [warp][4 rows][F + 1] when phi_in_smem
    __shared__ uint32_t s_feat[kShapQWarps][kShapQFrames];  // split feature of each frame (uniform)
    const uint32_t F = m.n_features;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 3, pt = lane & 7;
    const float xi = c_rule_nodes[pt], wi = c_rule_weights[pt];
    const float f0 = c_f0[pt], r0 = c_r0[pt];
    float fc[kShapQFrames], fhl[kShapQFrames], fwp[kShapQFrames], fpe[kShapQFrames], fre[kShapQFrames];
    uint32_t fidx[kShapQFrames], fstage[kShapQFrames];
    const uint64_t step = (uint64_t)gridDim.x * kShapQWarps * 4;
    for (uint64_t base = ((uint64_t)blockIdx.x * kShapQWarps + warp) * 4; base < n; base += step) {
        const uint64_t r = base + g;
        const bool valid = r < n;
        const uint64_t rr = valid ? r : n - 1;
        const float* x = X + rr * F;
        float* phi = phi_in_smem ? sphi + (size_t)(warp * 4 + g) * (F + 1) : out + rr * (F + 1);
        if (valid || phi_in_smem)
            for (uint32_t f = pt; f <= F; f += 8) phi[f] = 0.0f;
        __syncwarp();
        for (uint32_t t = 0; t < m.n_trees; t++) {
            const uint32_t gb = m.tree_off[t];
            const DevNode* nodes = m.nodes + gb;
            if ((nodes[0].meta >> 24) & kNodeLeaf) continue;
            int sp = 0;
            fc[0] = 1.0f;
            fwp[0] = 1.0f;
            fidx[0] = 0;
            fstage[0] = 0;
            float h = 0.0f;
            bool have_ret = false;
            while (sp >= 0) {
                const uint32_t idx = fidx[sp];
                const DevNode nd = nodes[idx];
                const uint32_t feat = nd.meta & 0xffffffu;
                // the path probability before this node's edge: deepest ancestor on the same feature
                int anc = -1;
                for (int k = sp - 1; k >= 0; k--)
                    if (s_feat[warp][k] == feat) { anc = k; break; }
                const bool seen = anc >= 0;
                const float p_old = seen ? fpe[anc] : 1.0f;
                const float r_old = seen ? fre[anc] : 1.0f;
                if (have_ret) {
                    // return from the edge taken in fstage[sp]: explain.rs:345-349 + extract_delta
                    const float pe = fpe[sp];
                    float acc = 0.0f;
                    if (pe != 1.0f) acc = __fmul_rn(__fmul_rn(__fsub_rn(pe, 1.0f), h), fre[sp]);
                    if (seen && p_old != 1.0f)
                        acc = __fsub_rn(acc, __fmul_rn(__fmul_rn(__fsub_rn(p_old, 1.0f), h), r_old));
                    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
                    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
                    if (pt == 0 && (valid || phi_in_smem)) phi[feat] += acc;
                    if (fstage[sp] == 0) {
                        fhl[sp] = h;
                        fstage[sp] = 1;
                        have_ret = false;
                    } else {
                        h = __fadd_rn(fhl[sp], h);
                        sp--;
                        continue;  // have_ret stays true for the parent frame
                    }
                }
                // take the edge of fstage[sp]: explain.rs:312-350 visit_child
                const bool left_side = fstage[sp] == 0;
                const int32_t child = left_side ? nd.left : nd.right;
                const uint32_t cg = gb + (uint32_t)child;
                const float2 ew = e.w[cg];  // (cw, 1 / cw)
                const bool gl = node_goes_left(nd, m, gb + idx, x[feat]);
                const bool sat = left_side ? gl : !gl;
                float pe, fe, re;
                if (!sat) {
                    pe = 0.0f; fe = f0; re = r0;
                } else if (!seen) {
                    pe = ew.y; fe = e.f[cg * kShapPoints + pt]; re = e.r[cg * kShapPoints + pt];
                } else {
                    pe = __fdiv_rn(p_old, ew.x);
                    fe = __fadd_rn(1.0f, __fmul_rn(__fsub_rn(pe, 1.0f), xi));
                    re = __fdividef(1.0f, fe);
                }
                float cc = __fmul_rn(fc[sp], fe);
                if (seen && p_old != 1.0f) cc = __fmul_rn(cc, r_old);
                fpe[sp] = pe;
                fre[sp] = re;
                if (lane == 0) s_feat[warp][sp] = feat;
                __syncwarp();
                const float wpc = __fmul_rn(fwp[sp], ew.x);
                const DevNode ch = nodes[child];
                if ((ch.meta >> 24) & kNodeLeaf) {
                    h = __fmul_rn(__fmul_rn(cc, __fmul_rn(wpc, ch.val)), wi);
                    have_ret = true;
                } else {
                    sp++;
                    fc[sp] = cc;
                    fwp[sp] = wpc;
                    fidx[sp] = (uint32_t)child;
                    fstage[sp] = 0;
                }
            }
        }
        if (pt == 0 && (valid || phi_in_smem)) phi[F] = __fadd_rn(__fadd_rn(phi[F], root_mean), bias);
        __syncwarp();
        if (phi_in_smem && valid)
            for (uint32_t f = pt; f <= F; f += 8) out[rr * (F + 1) + f] = phi[f];
        __syncwarp();
    }
}

void upload_shap_rule(const float* nodes, const float* weights, cudaStream_t s) {
    cudaMemcpyToSymbolAsync(c_rule_nodes, nodes, sizeof(float) * kShapPoints, 0, cudaMemcpyHostToDevice, s);
    cudaMemcpyToSymbolAsync(c_rule_weights, weights, sizeof(float) * kShapPoints, 0, cudaMemcpyHostToDevice, s);
    float f0[kShapPoints], r0[kShapPoints];
    for (int i = 0; i < kShapPoints; i++) {
        f0[i] = 1.0f + (-1.0f) * nodes[i];  // alpha = p_e - 1 = -1
        r0[i] = 1.0f / f0[i];
    }
    cudaMemcpyToSymbolAsync(c_f0, f0, sizeof(f0), 0, cudaMemcpyHostToDevice, s);
    cudaMemcpyToSymbolAsync(c_r0, r0, sizeof(r0), 0, cudaMemcpyHostToDevice, s);
}

bool shap_q_supported(const DevModel& m) { return m.max_depth <= kMaxShapDepth; }

void launch_shap_q(const DevModel& m, const ShapEdges& e, const float* X, uint64_t n, float bias, float root_mean,
                   float* out, cudaStream_t s) {
    if (n == 0) return;
    const uint32_t F = m.n_features;
    const size_t smem = (size_t)kShapQWarps * 4 * (F + 1) * sizeof(float);
    const uint32_t in_smem = smem <= 48 * 1024 ? 1u : 0u;
    uint64_t blocks = (n + 4 * kShapQWarps - 1) / (4 * kShapQWarps);
    if (blocks > 148ull * 32) blocks = 148ull * 32;
    count_launch();
    k_shap_q<<<(unsigned)blocks, 32 * kShapQWarps, in_smem ? smem : 0, s>>>(m, e, X, n, bias, root_mean, out, in_smem);
}

void launch_predict(const DevModel& m, const float* X, uint64_t n, float base_margin, float* out, cudaStream_t s) {
    if (n == 0) return;
    uint64_t blocks = (n + 255) / 256;
    if (blocks > 148ull * 64) blocks = 148ull * 64;
    count_launch();
    k_predict<<<(unsigned)blocks, 256, 0, s>>>(m, X, n, base_margin, out);
}

// Rows in flight: each thread's DFS frames (up to 15 x 84 B) live in local
// memory, so the resident threads are capped to keep that working set in L1
// (FBGPU_SHAP_CTAS_PER_SM overrides the cap of 128-thread CTAs per SM).
uint64_t shap_threads(uint64_t n) {
    static const uint64_t per_sm = [] {
        const char* v = std::getenv("FBGPU_SHAP_CTAS_PER_SM");
        const long k = v ? std::atol(v) : 0;
        return (uint64_t)(k > 0 && k <= 64 ? k : 16);
    }();
    uint64_t t = ((n + 127) / 128) * 128;
    const uint64_t cap = 148ull * per_sm * 128;
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
