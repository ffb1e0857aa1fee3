// Process-wide cache of device blocks behind DevMem.
//
// A training call allocates several gigabytes (row records, the column copy,
// the sketch's work space, gradients, histograms) and frees them when it
// returns.  Supplying fresh device memory is not always cheap: on B200 a
// cudaMalloc / cudaFree of that size occasionally took hundreds of
// milliseconds, which showed up as one-second outliers in the end-to-end
// timing of repeated trainings.  Blocks are therefore kept per device when
// released (sizes from 1 MiB rounded to 2 MiB, smaller ones to a power of
// two) and handed to the next allocation they fit (at most 1.5 x its size,
// so a large block is not spent on a small request).  A block is cached
// only after its device has finished all work (the synchronisation cudaFree
// itself implies), the cache holds at most a quarter of the device's memory,
// and an allocation that fails empties the cache and tries again.  Pinned
// host buffers are kept the same way (pinned_alloc / pinned_free, power-of-two
// sizes, up to 1 GiB in all).
#include <cuda_runtime.h>

#include <map>
#include <mutex>

#include "ctx.h"

namespace fbg {
namespace {

constexpr size_t kLarge = 1ull << 20;
constexpr size_t kRound = 2ull << 20;
constexpr int kMaxDevices = 64;

struct BlockCache {
    std::mutex mu;
    std::multimap<size_t, void*> free[kMaxDevices];
    size_t held[kMaxDevices] = {};
    size_t limit[kMaxDevices] = {};
};

BlockCache& cache() {
    static BlockCache* c = new BlockCache;  // never destroyed: blocks may be released during static teardown
    return *c;
}

size_t rounded(size_t n) {
    if (n >= kLarge) return (n + kRound - 1) / kRound * kRound;
    size_t c = 512;
    while (c < n) c <<= 1;
    return c;
}

// Frees every cached block of `dev` (the caller holds the lock).
void drain(BlockCache& c, int dev) {
    for (auto& kv : c.free[dev]) cudaFree(kv.second);
    c.free[dev].clear();
    c.held[dev] = 0;
}

}  // namespace

void* dev_alloc(size_t n, size_t* cap) {
    const size_t want = rounded(n);
    int dev = 0;
    FB_CUDA_CHECK(cudaGetDevice(&dev));
    BlockCache& c = cache();
    if (dev >= 0 && dev < kMaxDevices) {
        std::lock_guard<std::mutex> lock(c.mu);
        auto& m = c.free[dev];
        auto it = m.lower_bound(want);
        if (it != m.end() && it->first <= want + want / 2) {
            void* p = it->second;
            *cap = it->first;
            c.held[dev] -= it->first;
            m.erase(it);
            return p;
        }
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e == cudaErrorMemoryAllocation && dev >= 0 && dev < kMaxDevices) {
        (void)cudaGetLastError();
        {
            std::lock_guard<std::mutex> lock(c.mu);
            drain(c, dev);
        }
        e = cudaMalloc(&p, want);
    }
    if (e != cudaSuccess) throw CudaError(e, "cudaMalloc", __FILE__, __LINE__);
    *cap = want;
    return p;
}

void dev_free(void* p, size_t cap) {
    if (!p) return;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || attr.type != cudaMemoryTypeDevice || attr.device < 0 ||
        attr.device >= kMaxDevices) {
        (void)cudaGetLastError();
        cudaFree(p);
        return;
    }
    const int dev = attr.device;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != dev) cudaSetDevice(dev);
    const cudaError_t sync = cudaDeviceSynchronize();  // as cudaFree: the device is done with the block
    if (cur != dev) cudaSetDevice(cur);
    BlockCache& c = cache();
    std::lock_guard<std::mutex> lock(c.mu);
    if (!c.limit[dev]) {
        size_t fr = 0, total = 0;
        if (cur != dev) cudaSetDevice(dev);
        if (cudaMemGetInfo(&fr, &total) != cudaSuccess) (void)cudaGetLastError();
        if (cur != dev) cudaSetDevice(cur);
        c.limit[dev] = total / 4;
    }
    if (sync != cudaSuccess || c.held[dev] + cap > c.limit[dev]) {
        cudaFree(p);
        return;
    }
    c.free[dev].emplace(cap, p);
    c.held[dev] += cap;
}

namespace {
struct HostCache {
    std::mutex mu;
    std::multimap<size_t, void*> free;
    size_t held = 0;
};
HostCache& host_cache() {
    static HostCache* c = new HostCache;
    return *c;
}
constexpr size_t kHostCacheLimit = 1ull << 30;
}  // namespace

void* pinned_alloc(size_t n, size_t* cap) {
    size_t want = 4096;
    while (want < n) want <<= 1;
    HostCache& c = host_cache();
    {
        std::lock_guard<std::mutex> lock(c.mu);
        auto it = c.free.find(want);
        if (it != c.free.end()) {
            void* p = it->second;
            c.free.erase(it);
            c.held -= want;
            *cap = want;
            return p;
        }
    }
    void* p = nullptr;
    FB_CUDA_CHECK(cudaMallocHost(&p, want));
    *cap = want;
    return p;
}

void pinned_free(void* p, size_t cap) {
    if (!p) return;
    // as cudaFreeHost: no copy into or out of the buffer is still in flight
    if (cudaDeviceSynchronize() != cudaSuccess) {
        (void)cudaGetLastError();
        cudaFreeHost(p);
        return;
    }
    HostCache& c = host_cache();
    std::lock_guard<std::mutex> lock(c.mu);
    if (c.held + cap > kHostCacheLimit) {
        cudaFreeHost(p);
        return;
    }
    c.free.emplace(cap, p);
    c.held += cap;
}

}  // namespace fbg
