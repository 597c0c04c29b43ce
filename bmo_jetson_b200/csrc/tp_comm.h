// tp_comm.h -- the collective of the tensor-parallel batch-1 mode: NCCL,
// loaded at run time (libnccl.so.2) so that libbmo.so has no link-time NCCL
// dependency and shares the NCCL a host process (e.g. PyTorch) already loaded.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace bmo {

constexpr int kTpIdBytes = 128;  // NCCL unique id

class TpComm {
public:
    // Joins rank `rank` of `size` ranks identified by `id` (from tp_unique_id
    // on one rank, passed to all).  Throws with the NCCL message on failure.
    TpComm(const void *id, int rank, int size);
    ~TpComm();
    TpComm(const TpComm &) = delete;
    TpComm &operator=(const TpComm &) = delete;
    // In-place sum of n doubles over the ranks, on stream s (capturable).
    void all_reduce_sum(double *buf, size_t n, cudaStream_t s);
    // Host-side setup collectives (synchronous): every rank's `bytes` bytes of
    // `send`, rank by rank, into `recv`; the minimum of v over the ranks;
    // a barrier.
    void all_gather_bytes(const void *send, void *recv, size_t bytes);
    int all_min(int v);
    void barrier() { (void)all_min(1); }
    int rank() const { return rank_; }
    int size() const { return size_; }

private:
    void *comm_ = nullptr;
    int rank_ = 0, size_ = 1;
};

// A fresh NCCL unique id (kTpIdBytes bytes) for one tensor-parallel group.
void tp_unique_id(void *out);
// Empty when NCCL can be loaded, else why not.
std::string tp_unavailable();

}  // namespace bmo
