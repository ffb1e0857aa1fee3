// NCCL communicator used by the row-sharded training.  The library has no
// link dependency on NCCL: the entry points are resolved at run time (dlopen),
// so a process shares the copy it already loaded (PyTorch loads libnccl.so.2;
// $FBGPU_NCCL_LIB names another file).  The communicator is non-blocking, and
// every wait on it is a host-side poll with a time limit that aborts the
// communicator (ending its kernels) when a peer does not answer.
#pragma once
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include <cuda_runtime.h>

namespace fbg {

constexpr int kNcclUniqueIdBytes = 128;  // NCCL_UNIQUE_ID_BYTES

struct NcclError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct TimeoutError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void nccl_unique_id(uint8_t* out);

class NcclComm {
public:
    // wait == false returns as soon as the non-blocking initialization has
    // started; wait_init() then completes it.
    NcclComm(const uint8_t* unique_id, int nranks, int rank, int device, uint32_t timeout_ms, bool wait = true);
    void wait_init() { wait_ready("ncclCommInitRankConfig"); }
    ~NcclComm();
    NcclComm(const NcclComm&) = delete;
    NcclComm& operator=(const NcclComm&) = delete;

    // In place when src == dst.  u64: ncclUint64 with sum or max; otherwise ncclUint32 sum.
    void allreduce(const void* src, void* dst, size_t count, bool u64, bool max_op, cudaStream_t s);
    // ncclReduceScatter (u64 sum): rank r receives the sum of block r (recv_count words) of every rank's src.
    void reduce_scatter_u64(const void* src, void* dst, size_t recv_count, cudaStream_t s);
    // ncclAllGather: dst holds every rank's send_bytes, in rank order.
    void all_gather_bytes(const void* src, void* dst, size_t send_bytes, cudaStream_t s);
    // Waits for the stream (or an event), polling the communicator; aborts it
    // after the time limit.
    void sync(cudaStream_t s);
    void wait_event(cudaEvent_t ev);
    bool failed() const { return failed_; }
    // Ends the communicator at once, without waiting for the peers (exit
    // paths; nothing may be in flight on it); later calls fail.
    void abort();

private:
    void* comm_ = nullptr;  // ncclComm_t
    uint32_t timeout_ms_;
    bool failed_ = false;
    void wait_ready(const char* what);  // until the last call is no longer in progress
    template <class Q> void wait(Q query);
    [[noreturn]] void fail(const std::string& msg, bool timeout);
};

}  // namespace fbg
