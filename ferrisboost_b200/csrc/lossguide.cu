// Best-first (lossguide) tree growth on the device when max_leaves binds
// (training/lossguide.rs:506-700).
//
// The reference pops one leaf at a time: the pending leaf with the largest
// gain (lower node id on ties) is split, its children are evaluated (the
// smaller one accumulated, the larger one its parent minus the smaller) and
// pushed.  Here the host replays exactly that pop order, and the device
// evaluates children in waves: when the next leaf to pop has not been
// expanded yet, the host expands it together with the next best pending
// leaves (at most as many as pops remain), in one batch of kernels.  A leaf
// expanded this way but never popped stays a leaf: its rows still fill its
// span, so only its children's evaluations were wasted.  Every popped leaf's
// expansion is the same arithmetic as the reference's, so the tree is the
// reference's tree bit for bit.
//
// Device state per tree: a slot table of evaluated nodes (NodeInfo span /
// sum / bounds, best split, categories), a pool of full node histograms
// (the larger child reuses its parent's slot, as hist::subtract_in_place
// does), and one row arena (rows_[0]); a wave partitions its nodes into
// rows_[1] and copies the spans back.
#include <algorithm>
#include <array>
#include <cfloat>
#include <cstring>
#include <vector>

#include "ctx.h"

namespace fbg {

struct WaveEntry {     // one expansion (host -> device)
    uint32_t slot;     // slot to split
    uint32_t child[2]; // slots of its children
    int32_t new_hist;  // pool slot for the smaller child's histogram; -1: children are not evaluated
};

struct WaveOut {       // one expansion (device -> host)
    float lv, rv;      // child leaf values (xgb_weight x eta, bounded by the parent's bounds)
    float lh, rh;      // child hessians
    uint32_t small;    // 0: the left child was accumulated, 1: the right one
    uint32_t pad[3];
};
static_assert(sizeof(WaveOut) == 32, "WaveOut layout");

struct LgArgs {
    NodeInfo* slots;
    int32_t* slot_hist;
    SplitRec* slot_best;
    uint32_t* slot_cats;
    const WaveEntry* wave;
    uint32_t n_wave;
    WaveOut* wave_out;
    uint32_t* eval_slot;
    uint32_t* node_hist;
    const uint32_t* final_slot;
    const float* final_value;
    uint32_t n_final;
};

namespace {

__device__ __forceinline__ uint32_t block_scan_u32_1024(uint32_t v, uint32_t* wt, uint32_t& total) {
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= (uint32_t)o) x += y;
    }
    if (lane == 31) wt[w] = x;
    __syncthreads();
    if (w == 0) {
        uint32_t t = lane < (blockDim.x >> 5) ? wt[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= (uint32_t)o) t += y;
        }
        wt[lane] = t;
    }
    __syncthreads();
    const uint32_t before = w ? wt[w - 1] : 0u;
    total = wt[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + x - v;
}

__device__ __forceinline__ unsigned long long block_scan_u64_1024(unsigned long long v, unsigned long long* wt,
                                                                   unsigned long long& total) {
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= (uint32_t)o) x += y;
    }
    if (lane == 31) wt[w] = x;
    __syncthreads();
    if (w == 0) {
        unsigned long long t = lane < (blockDim.x >> 5) ? wt[lane] : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            unsigned long long y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= (uint32_t)o) t += y;
        }
        wt[lane] = t;
    }
    __syncthreads();
    const unsigned long long before = w ? wt[w - 1] : 0ull;
    total = wt[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + x - v;
}

// After the root's k_tree_init (a.nodes = evaluation list): the root is slot 0
// with pool histogram 0.
__global__ void k_lg_root(LevelArgs a, LgArgs g) {
    if (threadIdx.x != 0) return;
    g.slots[0] = a.nodes[0];
    g.slot_hist[0] = 0;
    g.node_hist[0] = 0;
    g.eval_slot[0] = 0;
}

// Partition list of a wave: the expanded slots, their split descriptors and
// categories, and the chunk table (one CTA).
__global__ void __launch_bounds__(1024) k_wave_setup(LevelArgs a, LgArgs g) {
    __shared__ uint32_t wt[32];
    uint32_t carry = 0;
    for (uint32_t base = 0; base < g.n_wave; base += 1024) {
        const uint32_t k = base + threadIdx.x;
        uint32_t chunks = 0;
        if (k < g.n_wave) {
            const uint32_t s = g.wave[k].slot;
            const NodeInfo ni = g.slots[s];
            a.nodes[k] = ni;
            const SplitRec b = g.slot_best[s];
            a.split[k] = SplitDesc{(int32_t)(2 * k), b.feat, b.bin, b.flags & 6u};
            for (uint32_t w = 0; w < a.cat_words; w++)
                a.node_cats[(size_t)k * a.cat_words + w] = g.slot_cats[(size_t)s * a.cat_words + w];
            chunks = (ni.len + kChunkRows - 1) / kChunkRows;
        }
        uint32_t tot;
        const uint32_t ex = block_scan_u32_1024(chunks, wt, tot);
        if (k < g.n_wave) const_cast<uint32_t*>(a.chunk_prefix)[k] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) {
        const_cast<uint32_t*>(a.chunk_prefix)[g.n_wave] = carry;
        a.st->m = g.n_wave;
        a.st->chunk_count = carry;
    }
}

// Copy the partitioned spans of the wave (rows_next) back into the arena.
__global__ void __launch_bounds__(kPartThreads) k_wave_copy_back(LevelArgs a) {
    const uint32_t c = blockIdx.x;
    const TreeState* st = a.st;
    if (c >= st->chunk_count) return;
    const uint32_t m = st->m;
    uint32_t lo = 0, hi = m;  // last node whose first chunk <= c
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a.chunk_prefix[mid] <= c) lo = mid; else hi = mid;
    }
    const NodeInfo ni = a.nodes[lo];
    const uint32_t r0 = (c - a.chunk_prefix[lo]) * kChunkRows;
    const uint32_t cnt = min(kChunkRows, ni.len - r0);
    const uint32_t* src = a.rows_next + ni.start + r0;
    uint32_t* dst = const_cast<uint32_t*>(a.rows_cur) + ni.start + r0;
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) dst[i] = src[i];
}

// Children of every expanded slot (one CTA): spans from the partition counts,
// sums and monotone bounds from the split (training/mod.rs:5069-5093
// child_leaves; split.rs:140-153), leaf values for the host tree, and the
// evaluation list (smaller child by rows over all ranks, lossguide.rs:72-120).
__global__ void __launch_bounds__(1024) k_wave_children(LevelArgs a, LgArgs g) {
    __shared__ uint32_t wt[32];
    __shared__ unsigned long long wt64[32];
    const ScoreParams sp = load_sp(a);
    uint32_t eval_before = 0;
    for (uint32_t base = 0; base < g.n_wave; base += 1024) {
        const uint32_t k = base + threadIdx.x;
        const bool valid = k < g.n_wave;
        const bool evaluate = valid && g.wave[k].new_hist >= 0;
        uint32_t tot;
        const uint32_t rank = eval_before + block_scan_u32_1024(evaluate ? 1u : 0u, wt, tot);
        eval_before += tot;
        if (!valid) continue;
        const WaveEntry we = g.wave[k];
        const NodeInfo ni = a.nodes[k];
        const SplitRec b = g.slot_best[we.slot];
        const uint32_t nl = a.node_left[k], nr = ni.len - nl;
        const uint32_t nlg = a.node_left_global ? a.node_left_global[k] : 0u;
        const uint32_t nrg = a.node_left_global ? ni.len_global - nlg : 0u;
        const double lg = to_f64(b.left.g, sp.inv_g), lh = to_f64(b.left.h, sp.inv_h);
        const double rg = to_f64(b.right.g, sp.inv_g), rh = to_f64(b.right.h, sp.inv_h);
        const float wl = apply_bounds(xgb_weight(lg, lh, sp), ni.lower, ni.upper);
        const float wr = apply_bounds(xgb_weight(rg, rh, sp), ni.lower, ni.upper);
        const int cons = a.mono ? (int)a.mono[b.feat] : 0;
        const float mid = __fdiv_rn(__fadd_rn(wl, wr), 2.0f);
        float llo = ni.lower, lhi = ni.upper, rlo = ni.lower, rhi = ni.upper;
        if (cons < 0) { llo = mid; rhi = mid; } else if (cons > 0) { lhi = mid; rlo = mid; }
        NodeInfo L, R;
        L.start = ni.start; L.len = nl; L.len_global = nlg; L.sum = b.left; L.lower = llo; L.upper = lhi;
        R.start = ni.start + nl; R.len = nr; R.len_global = nrg; R.sum = b.right; R.lower = rlo; R.upper = rhi;
        L.tree_id = R.tree_id = -1;
        // by rows; row-sharded: by the children's global hessian sums
        const uint32_t small = a.node_left_global ? (nlg <= nrg ? 0u : 1u) : (b.left.h <= b.right.h ? 0u : 1u);
        WaveOut o;
        o.lv = __fmul_rn(wl, sp.eta);
        o.rv = __fmul_rn(wr, sp.eta);
        o.lh = __double2float_rn(lh);
        o.rh = __double2float_rn(rh);
        o.small = small;
        o.pad[0] = o.pad[1] = o.pad[2] = 0;
        g.wave_out[k] = o;
        const int32_t parent_hist = g.slot_hist[we.slot];
        if (evaluate) {
            const uint32_t e = 2 * rank;
            L.acc_slot = R.acc_slot = (int32_t)rank;
            L.parent_slot = small == 0 ? -1 : parent_hist;
            R.parent_slot = small == 1 ? -1 : parent_hist;
            a.next_nodes[e] = L;
            a.next_nodes[e + 1] = R;
            g.node_hist[e + small] = (uint32_t)we.new_hist;
            g.node_hist[e + 1 - small] = (uint32_t)parent_hist;
            g.eval_slot[e] = we.child[0];
            g.eval_slot[e + 1] = we.child[1];
            a.next_acc_list[rank] = e + small;
            g.slot_hist[we.child[small]] = we.new_hist;
            g.slot_hist[we.child[1 - small]] = parent_hist;
        } else {
            L.acc_slot = R.acc_slot = 0;
            L.parent_slot = R.parent_slot = -1;
            g.slot_hist[we.child[0]] = -1;
            g.slot_hist[we.child[1]] = -1;
        }
        g.slots[we.child[0]] = L;
        g.slots[we.child[1]] = R;
        g.slot_hist[we.slot] = -1;
    }
    __syncthreads();
    // row prefix of the accumulated children, for the histogram kernels
    const uint32_t n_eval = eval_before;
    unsigned long long carry = 0;
    for (uint32_t base = 0; base < n_eval; base += 1024) {
        const uint32_t k = base + threadIdx.x;
        const unsigned long long v = k < n_eval ? a.next_nodes[a.next_acc_list[k]].len : 0ull;
        unsigned long long tot;
        const unsigned long long ex = block_scan_u64_1024(v, wt64, tot);
        if (k < n_eval) a.next_acc_prefix[k] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) {
        a.next_acc_prefix[n_eval] = carry;
        a.st->m = 2 * n_eval;
        a.st->acc_count = n_eval;
        a.st->acc_total = carry;
    }
}

// Best splits of the evaluated children into their slots.
__global__ void k_wave_store(LevelArgs a, LgArgs g) {
    const uint32_t m = a.st->m;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) {
        const uint32_t s = g.eval_slot[i];
        g.slot_best[s] = a.node_best[i];
        for (uint32_t w = 0; w < a.cat_words; w++)
            g.slot_cats[(size_t)s * a.cat_words + w] = a.node_cats[(size_t)i * a.cat_words + w];
    }
}

// Final leaves of the tree: spans of their slots, values into trec[i].leaf,
// chunk table for k_leaf_final (one CTA).
__global__ void __launch_bounds__(1024) k_final_setup(LevelArgs a, LgArgs g) {
    __shared__ uint32_t wt[32];
    uint32_t carry = 0;
    for (uint32_t base = 0; base < g.n_final; base += 1024) {
        const uint32_t i = base + threadIdx.x;
        uint32_t chunks = 0;
        if (i < g.n_final) {
            NodeInfo ni = g.slots[g.final_slot[i]];
            ni.tree_id = (int32_t)i;
            a.nodes[i] = ni;
            TreeRec t{-1, -1, 0, 0, 0.0f, g.final_value[i], 0.0f, 1u};
            a.trec[i] = t;
            chunks = (ni.len + kChunkRows - 1) / kChunkRows;
        }
        uint32_t tot;
        const uint32_t ex = block_scan_u32_1024(chunks, wt, tot);
        if (i < g.n_final) const_cast<uint32_t*>(a.chunk_prefix)[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) {
        const_cast<uint32_t*>(a.chunk_prefix)[g.n_final] = carry;
        a.st->m = g.n_final;
        a.st->chunk_count = carry;
    }
}

}  // namespace

// ----------------------------------------------------------------- host side
namespace {

struct HostSlot {
    uint32_t depth = 0;
    int32_t tree_id = -1;
    bool found = false;
    bool expanded = false;
    float gain = 0.0f;
    SplitRec best{};
    std::vector<uint32_t> cats;  // right-going set (cat_words words) of a categorical best split
    uint32_t child[2] = {0, 0};
    float cvalue[2] = {0, 0}, chess[2] = {0, 0};
    float value = 0.0f;  // own leaf value (set when its parent is split)
    int32_t hist = -1;   // pool histogram held by this slot
};

int32_t total_key(float g) {
    int32_t i;
    std::memcpy(&i, &g, 4);
    return i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
}

}  // namespace

void TrainCtx::build_tree_lossguide(const fbgpu_tree_params& tp, const uint8_t* enabled, fbgpu_tree_out* out) {
    const uint32_t max_leaves = tp.max_leaves, max_depth = tp.max_depth;
    LevelArgs a = level_args(tp);
    set_split_lists(a);
    a.last_level = 0;
    Pair* pool = hist_[0].as<Pair>();
    a.hist_cur = pool;
    a.hist_prev = pool;
    a.node_hist = lg_node_hist_.as<uint32_t>();
    a.acc_list = acc_list_[0].as<uint32_t>();
    a.acc_prefix = acc_prefix_[0].as<unsigned long long>();
    a.next_acc_list = acc_list_[0].as<uint32_t>();
    a.next_acc_prefix = acc_prefix_[0].as<unsigned long long>();
    a.chunk_prefix = chunk_prefix_[0].as<uint32_t>();
    a.rows_cur = rows_[0].as<uint32_t>();
    a.rows_next = rows_[1].as<uint32_t>();
    LgArgs g{};
    g.slots = lg_slots_.as<NodeInfo>();
    g.slot_hist = lg_slot_hist_.as<int32_t>();
    g.slot_best = lg_slot_best_.as<SplitRec>();
    g.slot_cats = lg_slot_cats_.as<uint32_t>();
    g.wave = lg_wave_.as<WaveEntry>();
    g.wave_out = lg_wave_out_.as<WaveOut>();
    g.eval_slot = lg_eval_slot_.as<uint32_t>();
    g.node_hist = lg_node_hist_.as<uint32_t>();
    g.final_slot = lg_final_slot_.as<uint32_t>();
    g.final_value = lg_final_value_.as<float>();
    NodeInfo* eval_nodes = nodes_[1].as<NodeInfo>();  // children being evaluated
    NodeInfo* part_nodes = nodes_[0].as<NodeInfo>();  // slots being partitioned / final leaves
    const uint32_t n_slots_cap = lg_slot_cap_, n_hist_cap = lg_hist_cap_;

    // pinned host staging: wave descriptors, results
    uint8_t* hp = h_lg_.as<uint8_t>();
    WaveEntry* h_wave = reinterpret_cast<WaveEntry*>(hp);
    WaveOut* h_out = reinterpret_cast<WaveOut*>(h_wave + lg_kmax_);
    SplitRec* h_best = reinterpret_cast<SplitRec*>(h_out + lg_kmax_);
    uint32_t* h_cats = reinterpret_cast<uint32_t*>(h_best + 2 * lg_kmax_);
    const uint32_t W = cat_words_;
    TreeRec* h_root = reinterpret_cast<TreeRec*>(h_cats + 2ull * W * lg_kmax_);
    uint32_t* h_fslot = reinterpret_cast<uint32_t*>(h_root + 1);
    float* h_fval = reinterpret_cast<float*>(h_fslot + max_leaves + 1);

    std::vector<HostSlot> slots(1);
    std::vector<int32_t> free_hist;
    for (int32_t i = (int32_t)n_hist_cap - 1; i >= 1; i--) free_hist.push_back(i);

    // evaluate the children listed in eval_nodes (m of them) and read them back
    auto evaluate = [&](uint32_t n_acc, uint32_t m) {
        FB_CUDA_CHECK(cudaMemsetAsync(hist_acc_.p, 0, 16ull * a.slot_pairs * n_acc, s_));
        a.nodes = eval_nodes;
        const bool root_rides = root_pending_;  // only at the root: the round's sum rides along
        if (root_rides)
            FB_CUDA_CHECK(cudaMemcpyAsync(hist_acc_.as<unsigned long long>() + 2ull * a.slot_pairs, sums_.p, 16,
                                          cudaMemcpyDeviceToDevice, s_));
        launch_histograms(a.rows_cur, eval_nodes, a.acc_list, a.acc_prefix, n_);
        allreduce_u64(hist_acc_.p, 2ull * a.slot_pairs * n_acc + (root_rides ? 2 : 0), false);
        if (root_rides) {
            FB_CUDA_CHECK(cudaMemcpyAsync(sums_.p, hist_acc_.as<unsigned long long>() + 2ull * a.slot_pairs, 16,
                                          cudaMemcpyDeviceToDevice, s_));
            launch_tree_init(a, (uint32_t)n_, (uint32_t)cfg_.n_rows_global, sums_.as<unsigned long long>(), s_);
            count_launch();
            k_lg_root<<<1, 32, 0, s_>>>(a, g);
            root_pending_ = false;
        }
        launch_split(a, m, s_);
        count_launch();
        k_wave_store<<<ceil_div(m, 256), 256, 0, s_>>>(a, g);
        FB_CUDA_CHECK(cudaMemcpyAsync(h_best, node_best_.p, sizeof(SplitRec) * m, cudaMemcpyDeviceToHost, s_));
        if (has_cat_)
            FB_CUDA_CHECK(cudaMemcpyAsync(h_cats, node_cats_.p, 4ull * W * m, cudaMemcpyDeviceToHost, s_));
    };
    auto absorb = [&](uint32_t pos, uint32_t slot) {
        HostSlot& hs = slots[slot];
        hs.best = h_best[pos];
        hs.found = (hs.best.flags & 1u) != 0;
        hs.gain = hs.best.gain;
        if (has_cat_ && (hs.best.flags & 4u)) hs.cats.assign(h_cats + (size_t)W * pos, h_cats + (size_t)W * (pos + 1));
    };
    auto release = [&](HostSlot& hs) {
        if (hs.hist >= 0) free_hist.push_back(hs.hist);
        hs.hist = -1;
    };

    // ---- root: histogram, best split, leaf value
    FB_CUDA_CHECK(cudaEventRecord(ev0_, s_));
    launch_iota(rows_[0].as<uint32_t>(), (uint32_t)n_, s_);
    a.nodes = eval_nodes;
    a.acc_list = acc_list_[0].as<uint32_t>();
    launch_tree_init(a, (uint32_t)n_, (uint32_t)cfg_.n_rows_global, sums_.as<unsigned long long>(), s_);
    count_launch();
    k_lg_root<<<1, 32, 0, s_>>>(a, g);
    const bool root_only = max_depth == 0 || max_leaves == 1;
    if (root_only && root_pending_) {
        reduce_root_sum(true);
        launch_tree_init(a, (uint32_t)n_, (uint32_t)cfg_.n_rows_global, sums_.as<unsigned long long>(), s_);
    }
    if (!root_only) evaluate(1, 1);
    FB_CUDA_CHECK(cudaMemcpyAsync(h_root, trec_.p, sizeof(TreeRec), cudaMemcpyDeviceToHost, s_));
    unsigned long long* herr = h_small_.as<unsigned long long>() + 80;
    if (scale_err_pending_)
        FB_CUDA_CHECK(cudaMemcpyAsync(herr, sums_.as<unsigned long long>() + 6, 8, cudaMemcpyDeviceToHost, s_));
    sync();
    check_scale_error(herr);
    slots[0].hist = 0;
    slots[0].value = h_root->leaf;
    slots[0].tree_id = 0;
    if (!root_only) absorb(0, 0);
    std::vector<TreeRec> tree(1, *h_root);
    std::vector<std::vector<uint32_t>> tree_cats(1);
    struct E {
        int32_t key;
        int32_t id;
        uint32_t slot;
    };
    auto less = [](const E& x, const E& y) { return x.key != y.key ? x.key < y.key : x.id > y.id; };
    std::vector<E> heap;
    std::vector<std::pair<uint32_t, float>> finals;
    if (!root_only && slots[0].found) {
        heap.push_back({total_key(slots[0].gain), 0, 0});
        if (max_depth <= 1) release(slots[0]);  // children are final: no histogram needed
    } else {
        finals.push_back({0u, slots[0].value});
        release(slots[0]);
    }
    uint32_t leaf_count = 1;

    // ---- best-first loop
    while ((max_leaves == 0 || leaf_count < max_leaves) && !heap.empty()) {
        const E top = heap.front();
        if (!slots[top.slot].expanded) {
            // wave: the best pending slots not yet expanded, at most as many as pops remain
            std::vector<E> order(heap);
            std::sort(order.begin(), order.end(), [&](const E& x, const E& y) { return less(y, x); });
            const uint32_t remaining = max_leaves - leaf_count;
            uint32_t k = 0;
            for (const E& e : order) {
                if (k >= remaining || k >= lg_kmax_) break;
                HostSlot& hs = slots[e.slot];
                if (hs.expanded) continue;
                if (slots.size() + 2 > n_slots_cap) break;
                const bool eval_children = hs.depth + 1 < max_depth;
                int32_t nh = -1;
                if (eval_children) {
                    if (free_hist.empty() || hs.hist < 0) {
                        if (k == 0) throw std::runtime_error("lossguide histogram pool exhausted");
                        break;
                    }
                    nh = free_hist.back();
                    free_hist.pop_back();
                }
                WaveEntry we;
                we.slot = e.slot;
                we.child[0] = (uint32_t)slots.size();
                we.child[1] = we.child[0] + 1;
                we.new_hist = nh;
                slots.emplace_back();
                slots.emplace_back();
                HostSlot& hs2 = slots[e.slot];  // slots may have moved
                hs2.child[0] = we.child[0];
                hs2.child[1] = we.child[1];
                slots[we.child[0]].depth = slots[we.child[1]].depth = hs2.depth + 1;
                h_wave[k++] = we;
            }
            if (k == 0) throw std::runtime_error("lossguide wave is empty");
            FB_CUDA_CHECK(cudaMemcpyAsync(lg_wave_.p, h_wave, sizeof(WaveEntry) * k, cudaMemcpyHostToDevice, s_));
            g.n_wave = k;
            a.nodes = part_nodes;
            a.next_nodes = eval_nodes;
            count_launch();
            k_wave_setup<<<1, 1024, 0, s_>>>(a, g);
            const uint32_t max_chunks = ceil_div(std::max<uint64_t>(n_, 1), kChunkRows) + k;
            launch_part_count(a, max_chunks, s_);
            launch_part_scan(a, s_);
            launch_part_scatter(a, max_chunks, s_);
            count_launch();
            k_wave_copy_back<<<max_chunks, kPartThreads, 0, s_>>>(a);
            count_launch();
            k_wave_children<<<1, 1024, 0, s_>>>(a, g);
            uint32_t n_eval = 0;
            for (uint32_t i = 0; i < k; i++) n_eval += h_wave[i].new_hist >= 0 ? 1u : 0u;
            if (n_eval) evaluate(n_eval, 2 * n_eval);
            FB_CUDA_CHECK(cudaMemcpyAsync(h_out, lg_wave_out_.p, sizeof(WaveOut) * k, cudaMemcpyDeviceToHost, s_));
            sync();
            uint32_t e = 0;
            for (uint32_t i = 0; i < k; i++) {
                const WaveEntry& we = h_wave[i];
                HostSlot& p = slots[we.slot];
                p.expanded = true;
                p.cvalue[0] = h_out[i].lv;
                p.cvalue[1] = h_out[i].rv;
                p.chess[0] = h_out[i].lh;
                p.chess[1] = h_out[i].rh;
                slots[we.child[0]].value = h_out[i].lv;
                slots[we.child[1]].value = h_out[i].rv;
                if (we.new_hist >= 0) {
                    const uint32_t small = h_out[i].small;
                    slots[we.child[small]].hist = we.new_hist;
                    slots[we.child[1 - small]].hist = p.hist;
                    p.hist = -1;
                    for (int c = 0; c < 2; c++) {
                        absorb(e + c, we.child[c]);
                        HostSlot& ch = slots[we.child[c]];
                        // a histogram is kept only while the slot may still be expanded
                        // with evaluated children
                        if (!ch.found || ch.depth + 1 >= max_depth) release(ch);
                    }
                    e += 2;
                } else {
                    release(p);
                }
            }
            continue;
        }
        // pop
        std::pop_heap(heap.begin(), heap.end(), less);
        heap.pop_back();
        HostSlot& p = slots[top.slot];
        const int32_t l = (int32_t)tree.size(), r = l + 1;
        TreeRec& node = tree[p.tree_id];
        node.left = l;
        node.right = r;
        node.feat = p.best.feat;
        node.bin = p.best.bin;
        node.gain = p.best.gain;
        node.leaf = 0.0f;
        node.flags = ((p.best.flags & 2u) ? 2u : 0u) | ((p.best.flags & 4u) ? 4u : 0u);
        if (p.best.flags & 4u) tree_cats[p.tree_id] = p.cats;
        tree.push_back(TreeRec{-1, -1, 0, 0, 0.0f, p.cvalue[0], p.chess[0], 1u});
        tree.push_back(TreeRec{-1, -1, 0, 0, 0.0f, p.cvalue[1], p.chess[1], 1u});
        tree_cats.emplace_back();
        tree_cats.emplace_back();
        leaf_count++;
        const uint32_t c0 = p.child[0], c1 = p.child[1];
        const uint32_t depth = p.depth + 1;
        slots[c0].tree_id = l;
        slots[c1].tree_id = r;
        const bool children_final = depth == max_depth || leaf_count == max_leaves;
        for (uint32_t c : {c0, c1}) {
            HostSlot& ch = slots[c];
            if (children_final || !ch.found) {
                finals.push_back({c, ch.value});
                release(ch);
            } else {
                heap.push_back({total_key(ch.gain), ch.tree_id, c});
                std::push_heap(heap.begin(), heap.end(), less);
            }
        }
    }
    for (const E& e : heap) finals.push_back({e.slot, slots[e.slot].value});

    // ---- margins: each final leaf's value on the rows of its span
    const uint32_t nf = (uint32_t)finals.size();
    if (nf > max_leaves + 1) throw std::runtime_error("lossguide produced more leaves than max_leaves");
    for (uint32_t i = 0; i < nf; i++) {
        h_fslot[i] = finals[i].first;
        h_fval[i] = finals[i].second;
    }
    FB_CUDA_CHECK(cudaMemcpyAsync(lg_final_slot_.p, h_fslot, 4ull * nf, cudaMemcpyHostToDevice, s_));
    FB_CUDA_CHECK(cudaMemcpyAsync(lg_final_value_.p, h_fval, 4ull * nf, cudaMemcpyHostToDevice, s_));
    g.n_final = nf;
    a.nodes = part_nodes;
    count_launch();
    k_final_setup<<<1, 1024, 0, s_>>>(a, g);
    launch_leaf_final(a, ceil_div(std::max<uint64_t>(n_, 1), kChunkRows) + nf, s_);
    FB_CUDA_CHECK(cudaGetLastError());
    FB_CUDA_CHECK(cudaEventRecord(ev1_, s_));
    sync();
    FB_CUDA_CHECK(cudaEventElapsedTime(&last_tree_ms_, ev0_, ev1_));

    const uint32_t nn = (uint32_t)tree.size();
    if (!out) return;
    if (out->capacity < nn) throw InputError("fbgpu_tree_out capacity is smaller than the tree");
    const uint32_t out_w = out->cat_words ? out->cat_words : 8u;
    if (out->cats && out_w < W)
        throw InputError("fbgpu_tree_out.cat_words is smaller than the context's category sets (fbgpu_ctx_cat_words)");
    out->n_nodes = nn;
    for (uint32_t i = 0; i < nn; i++) {
        const TreeRec& t = tree[i];
        if (out->left) out->left[i] = t.left;
        if (out->right) out->right[i] = t.right;
        if (out->feat) out->feat[i] = t.feat;
        if (out->bin) out->bin[i] = t.bin;
        if (out->gain) out->gain[i] = t.gain;
        if (out->leaf) out->leaf[i] = t.leaf;
        if (out->hess) out->hess[i] = t.hess;
        if (out->flags) out->flags[i] = t.flags;
        if (out->cats)
            for (uint32_t w = 0; w < out_w; w++)
                out->cats[(size_t)i * out_w + w] = w < tree_cats[i].size() ? tree_cats[i][w] : 0u;
    }
    (void)enabled;
}

void TrainCtx::ensure_lossguide_buffers(uint32_t max_leaves) {
    if (lg_leaves_ == max_leaves) return;
    lg_kmax_ = max_leaves;
    lg_slot_cap_ = 4 * max_leaves + 8;
    lg_hist_cap_ = 2 * max_leaves + 4;
    lg_slots_.alloc(sizeof(NodeInfo) * lg_slot_cap_);
    lg_slot_hist_.alloc(4ull * lg_slot_cap_);
    lg_slot_best_.alloc(sizeof(SplitRec) * lg_slot_cap_);
    lg_slot_cats_.alloc(4ull * cat_words_ * lg_slot_cap_);
    FB_CUDA_CHECK(cudaMemsetAsync(lg_slot_cats_.p, 0, lg_slot_cats_.bytes, s_));
    lg_wave_.alloc(sizeof(WaveEntry) * lg_kmax_);
    lg_wave_out_.alloc(sizeof(WaveOut) * lg_kmax_);
    lg_eval_slot_.alloc(4ull * 2 * lg_kmax_);
    lg_node_hist_.alloc(4ull * 2 * lg_kmax_);
    lg_final_slot_.alloc(4ull * (max_leaves + 1));
    lg_final_value_.alloc(4ull * (max_leaves + 1));
    h_lg_.reserve(sizeof(WaveEntry) * lg_kmax_ + sizeof(WaveOut) * lg_kmax_ + sizeof(SplitRec) * 2 * lg_kmax_ +
                  8ull * cat_words_ * lg_kmax_ + sizeof(TreeRec) + 8ull * (max_leaves + 1) + 64);
    lg_leaves_ = max_leaves;
}

}  // namespace fbg
