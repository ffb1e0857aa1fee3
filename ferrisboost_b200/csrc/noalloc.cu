// Stable row partition that allocates no device memory.
//
// fbgpu_partition_noalloc runs the same count / scan / scatter kernels as the
// training context's partition (train_kernels.cu), but their scratch (the
// per-chunk left counts and offsets, and the one-node descriptor tables) lives
// in the fixed-size static device array below instead of context buffers.
// It is for callers that own every device allocation themselves and cannot
// call cudaMalloc (the reference's own Rust host keeps all allocation and
// lifetime on its side); they pass device pointers for the bins, the rows and
// the outputs, and nothing else is allocated.
//
// The array is shared by every call in the process on a given device and keeps
// the last call's contents; each call rewrites every part it reads before
// reading it.  Two calls whose kernels overlap on the GPU (different streams,
// or different host threads without ordering) race on it.
#include <cuda.h>  // CUcontext and the driver entry-point types (resolved at run time, no -lcuda)

#include <mutex>

#include "ctx.h"

namespace fbg {
namespace {

// Largest partition one call accepts: kNoAllocMaxChunks chunks of kChunkRows rows.
constexpr uint32_t kNoAllocMaxChunks = 65536;
constexpr uint64_t kNoAllocMaxRows = (uint64_t)kNoAllocMaxChunks * kChunkRows;  // 268,435,456

struct NoAllocScratch {
    TreeState st;
    NodeInfo node;
    SplitDesc split;
    FeatLoc floc;
    uint32_t chunk_prefix[2];
    uint32_t cats[8];
    uint32_t chunk_left[kNoAllocMaxChunks];
    uint32_t chunk_off[kNoAllocMaxChunks];
};

// 512 KiB + a few hundred bytes per device, held until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoAllocScratch)];

// The current context's process-unique id (cuCtxGetId, found through the
// runtime so the library needs no link to libcuda), or 0 when the driver
// offers no such call.  A context made after cudaDeviceReset gets a new id.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
        (void)cudaGetLastError();
    });
    if (!get_current || !get_id) return 0;
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (get_current(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

std::mutex g_mu;
struct CachedAddr {
    void* p = nullptr;
    unsigned long long ctx_id = 0;
};
CachedAddr g_addr[64];

// Device address of the scratch array on the current device, looked up with
// cudaGetSymbolAddress the first time a device (and context) is seen; the
// host-side name of the array is only a stand-in for the symbol.  The cache
// is keyed by the context's id, so a context made after cudaDeviceReset is
// looked up again instead of reusing a stale address.
NoAllocScratch* scratch_on(int device) {
    if (device < 0 || device >= 64) throw InputError("device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    CachedAddr& c = g_addr[device];
    const unsigned long long id = c.p ? current_context_id() : 0;
    if (!c.p || (id != 0 && id != c.ctx_id)) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) throw CudaError(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
        c.p = p;
        c.ctx_id = current_context_id();  // the lookup above made the context current
    }
    return static_cast<NoAllocScratch*>(c.p);
}

struct InitArgs {
    uint32_t n;
    uint32_t bin;
    uint32_t flags;
    uint32_t cats[8];
    FeatLoc floc;
};

// Writes every descriptor the partition kernels read (one node holding all n
// rows, split on feature slot 0).
__global__ void k_noalloc_init(NoAllocScratch* s, InitArgs a) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    TreeState st{};
    st.m = 1;
    st.chunk_count = (a.n + kChunkRows - 1) / kChunkRows;
    s->st = st;
    NodeInfo nd{};
    nd.start = 0;
    nd.len = a.n;
    nd.parent_slot = -1;
    s->node = nd;
    s->split = SplitDesc{0, 0u, a.bin, a.flags};
    s->floc = a.floc;
    s->chunk_prefix[0] = 0;
    s->chunk_prefix[1] = st.chunk_count;
    for (int w = 0; w < 8; w++) s->cats[w] = a.cats[w];
}

}  // namespace
}  // namespace fbg

extern "C" fbgpu_status fbgpu_partition_noalloc(const void* bins, uint32_t stride, uint32_t width, uint32_t byte_off,
                                                uint32_t missing_bin, const uint32_t* rows, uint64_t n, uint32_t bin,
                                                int32_t missing_left, const uint32_t* cats, uint32_t* out_rows,
                                                uint32_t* n_left, void* stream) {
    using namespace fbg;
    try {
        if (width != 1 && width != 2) throw InputError("bin width must be 1 or 2 bytes");
        if ((uint64_t)byte_off + width > stride) throw InputError("the feature lies outside the row record");
        // a two-byte bin is one 16-bit load: the records' base, stride and offset must keep it aligned
        if ((((uintptr_t)bins | stride | byte_off) & (width - 1)) != 0)
            throw InputError("two-byte bins need an even records address, stride and byte offset");
        if (n > kNoAllocMaxRows || n > 0xffffffffull)
            throw InputError("fbgpu_partition_noalloc accepts at most 268435456 rows per call");
        if (!n_left) throw InputError("n_left must be a device pointer");
        if (((uintptr_t)n_left | (uintptr_t)rows | (uintptr_t)out_rows) & 3u)
            throw InputError("rows, out_rows and n_left must be 4-byte aligned");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int device = 0;
        cudaError_t e = cudaGetDevice(&device);
        if (e != cudaSuccess) throw CudaError(e, "cudaGetDevice", __FILE__, __LINE__);
        if (s != nullptr && s != cudaStreamPerThread && s != cudaStreamLegacy) {
            int sdev = -1;
            e = cudaStreamGetDevice(s, &sdev);
            if (e != cudaSuccess) throw CudaError(e, "cudaStreamGetDevice", __FILE__, __LINE__);
            if (sdev != device) throw InputError("the stream belongs to another device than the current one");
        }
        if (n == 0) {
            e = cudaMemsetAsync(n_left, 0, sizeof(uint32_t), s);
            if (e != cudaSuccess) throw CudaError(e, "cudaMemsetAsync", __FILE__, __LINE__);
            return FBGPU_OK;
        }
        if (!bins || !rows || !out_rows) throw InputError("bins, rows and out_rows must be device pointers");
        // the scatter pass writes out_rows while other CTAs still read rows
        const uintptr_t r0 = (uintptr_t)rows, r1 = r0 + 4 * n, o0 = (uintptr_t)out_rows, o1 = o0 + 4 * n;
        if (r0 < o1 && o0 < r1) throw InputError("rows and out_rows must not overlap");
        NoAllocScratch* scr = scratch_on(device);
        InitArgs ia{};
        ia.n = (uint32_t)n;
        ia.bin = bin;
        ia.flags = (missing_left ? 2u : 0u) | (cats ? 4u : 0u);
        if (cats)
            for (int w = 0; w < 8; w++) ia.cats[w] = cats[w];
        ia.floc = FeatLoc{static_cast<const uint8_t*>(bins), stride, byte_off, width, missing_bin};
        count_launch();
        k_noalloc_init<<<1, 32, 0, s>>>(scr, ia);
        LevelArgs a{};
        a.st = &scr->st;
        a.nodes = &scr->node;
        a.split = &scr->split;
        a.floc = &scr->floc;
        a.chunk_prefix = scr->chunk_prefix;
        a.node_cats = scr->cats;
        a.cat_words = 8;
        a.chunk_left = scr->chunk_left;
        a.chunk_off = scr->chunk_off;
        a.node_left = n_left;
        a.rows_cur = rows;
        a.rows_next = out_rows;
        const uint32_t chunks = (uint32_t)((n + kChunkRows - 1) / kChunkRows);
        launch_part_count(a, chunks, s);
        launch_part_scan(a, s);
        launch_part_scatter(a, chunks, s);
        e = cudaGetLastError();
        if (e != cudaSuccess) throw CudaError(e, "partition launch", __FILE__, __LINE__);
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
