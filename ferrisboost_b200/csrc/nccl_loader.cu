// Run-time binding of the NCCL calls the row-sharded training uses, with
// bounded host-side waits (non-blocking communicator + ncclCommGetAsyncError).
#include "nccl_loader.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

namespace fbg {
namespace {

struct Api {
    void* handle = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_config = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclCommFinalize) finalize = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclReduceScatter) reduce_scatter = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    std::string why;
};

template <class T> void bind(void* h, T& fn, const char* name, std::string& why) {
    fn = reinterpret_cast<T>(dlsym(h, name));
    if (!fn && why.empty()) why = std::string("the loaded NCCL library lacks ") + name;
}

const Api& api() {
    static Api a = [] {
        Api r;
        const char* names[3] = {std::getenv("FBGPU_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
        for (const char* n : names) {
            if (!n || !*n) continue;
            r.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (r.handle) break;
        }
        if (!r.handle) {
            r.why = "NCCL library not found (import torch first, or set FBGPU_NCCL_LIB)";
            return r;
        }
        bind(r.handle, r.get_unique_id, "ncclGetUniqueId", r.why);
        bind(r.handle, r.init_config, "ncclCommInitRankConfig", r.why);
        bind(r.handle, r.async_error, "ncclCommGetAsyncError", r.why);
        bind(r.handle, r.finalize, "ncclCommFinalize", r.why);
        bind(r.handle, r.destroy, "ncclCommDestroy", r.why);
        bind(r.handle, r.abort, "ncclCommAbort", r.why);
        bind(r.handle, r.all_reduce, "ncclAllReduce", r.why);
        bind(r.handle, r.reduce_scatter, "ncclReduceScatter", r.why);
        bind(r.handle, r.all_gather, "ncclAllGather", r.why);
        bind(r.handle, r.error_string, "ncclGetErrorString", r.why);
        return r;
    }();
    if (!a.why.empty()) throw NcclError(a.why);
    return a;
}

std::string nccl_msg(const char* what, ncclResult_t rc) {
    return std::string("NCCL ") + what + ": " + api().error_string(rc);
}

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

}  // namespace

void nccl_unique_id(uint8_t* out) {
    ncclUniqueId id;
    const ncclResult_t rc = api().get_unique_id(&id);
    if (rc != ncclSuccess) throw NcclError(nccl_msg("ncclGetUniqueId", rc));
    std::memcpy(out, id.internal, kNcclUniqueIdBytes);
}

NcclComm::NcclComm(const uint8_t* unique_id, int nranks, int rank, int device, uint32_t timeout_ms, bool wait)
    : timeout_ms_(timeout_ms ? timeout_ms : 120000u) {
    static_assert(sizeof(ncclUniqueId) == kNcclUniqueIdBytes, "ncclUniqueId size");
    const Api& a = api();
    if (cudaSetDevice(device) != cudaSuccess) throw NcclError("cudaSetDevice failed before ncclCommInitRankConfig");
    ncclUniqueId id;
    std::memcpy(id.internal, unique_id, kNcclUniqueIdBytes);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t c = nullptr;
    const ncclResult_t rc = a.init_config(&c, nranks, id, rank, &cfg);
    comm_ = c;
    if (rc != ncclSuccess && rc != ncclInProgress) {
        if (c) a.abort(c);
        comm_ = nullptr;
        throw NcclError(nccl_msg("ncclCommInitRankConfig", rc));
    }
    if (wait) wait_ready("ncclCommInitRankConfig");
}

NcclComm::~NcclComm() {
    if (!comm_) return;
    const Api& a = api();
    ncclComm_t c = static_cast<ncclComm_t>(comm_);
    if (!failed_) {
        // flush, then destroy; a peer that never finalizes ends in an abort
        ncclResult_t rc = a.finalize(c);
        const auto t0 = Clock::now();
        while (rc == ncclInProgress && ms_since(t0) < timeout_ms_) {
            std::this_thread::yield();
            a.async_error(c, &rc);
        }
        if (rc == ncclSuccess) {
            a.destroy(c);
            return;
        }
    }
    a.abort(c);
}

void NcclComm::abort() {
    if (comm_ && !failed_) api().abort(static_cast<ncclComm_t>(comm_));
    comm_ = nullptr;
    failed_ = true;
}

void NcclComm::fail(const std::string& msg, bool timeout) {
    // abort ends the communicator's kernels still waiting on a peer
    if (comm_ && !failed_) api().abort(static_cast<ncclComm_t>(comm_));
    comm_ = nullptr;
    failed_ = true;
    if (timeout) throw TimeoutError(msg);
    throw NcclError(msg);
}

void NcclComm::wait_ready(const char* what) {
    const Api& a = api();
    ncclComm_t c = static_cast<ncclComm_t>(comm_);
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t rc = a.async_error(c, &st);
        if (rc != ncclSuccess) fail(nccl_msg("ncclCommGetAsyncError", rc), false);
        if (st == ncclSuccess) return;
        if (st != ncclInProgress) fail(nccl_msg(what, st), false);
        if (ms_since(t0) > timeout_ms_)
            fail(std::string("NCCL ") + what + ": no answer from a peer within " + std::to_string(timeout_ms_) + " ms",
                 true);
        std::this_thread::yield();
    }
}

void NcclComm::allreduce(const void* src, void* dst, size_t count, bool u64, bool max_op, cudaStream_t s) {
    if (failed_) throw NcclError("the NCCL communicator was aborted by an earlier error");
    const ncclResult_t rc = api().all_reduce(src, dst, count, u64 ? ncclUint64 : ncclUint32, max_op ? ncclMax : ncclSum,
                                             static_cast<ncclComm_t>(comm_), s);
    if (rc != ncclSuccess && rc != ncclInProgress) fail(nccl_msg("ncclAllReduce", rc), false);
    wait_ready("ncclAllReduce");
}

void NcclComm::reduce_scatter_u64(const void* src, void* dst, size_t recv_count, cudaStream_t s) {
    if (failed_) throw NcclError("the NCCL communicator was aborted by an earlier error");
    const ncclResult_t rc =
        api().reduce_scatter(src, dst, recv_count, ncclUint64, ncclSum, static_cast<ncclComm_t>(comm_), s);
    if (rc != ncclSuccess && rc != ncclInProgress) fail(nccl_msg("ncclReduceScatter", rc), false);
    wait_ready("ncclReduceScatter");
}

void NcclComm::all_gather_bytes(const void* src, void* dst, size_t send_bytes, cudaStream_t s) {
    if (failed_) throw NcclError("the NCCL communicator was aborted by an earlier error");
    const ncclResult_t rc =
        api().all_gather(src, dst, send_bytes, ncclUint8, static_cast<ncclComm_t>(comm_), s);
    if (rc != ncclSuccess && rc != ncclInProgress) fail(nccl_msg("ncclAllGather", rc), false);
    wait_ready("ncclAllGather");
}

template <class Q> void NcclComm::wait(Q query) {
    if (failed_) throw NcclError("the NCCL communicator was aborted by an earlier error");
    const Api& a = api();
    ncclComm_t c = static_cast<ncclComm_t>(comm_);
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t e = query();
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) {
            (void)cudaGetLastError();
            fail(std::string("CUDA error ") + cudaGetErrorString(e) + " while waiting for the NCCL stream", false);
        }
        ncclResult_t st = ncclSuccess;
        a.async_error(c, &st);
        if (st != ncclSuccess && st != ncclInProgress) fail(nccl_msg("asynchronous error", st), false);
        if (ms_since(t0) > timeout_ms_)
            fail("NCCL: a collective did not complete within " + std::to_string(timeout_ms_) +
                     " ms (a peer left or stalled); the communicator was aborted",
                 true);
        std::this_thread::yield();
    }
}

void NcclComm::sync(cudaStream_t s) { wait([s] { return cudaStreamQuery(s); }); }

void NcclComm::wait_event(cudaEvent_t ev) { wait([ev] { return cudaEventQuery(ev); }); }

}  // namespace fbg
