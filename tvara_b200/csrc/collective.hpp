// NCCL communicator for a tensor-parallel group.  libnccl is opened at run
// time (dlopen) so single-GPU use of the library never needs it; the few
// entry points used are resolved by name.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

namespace tvara {

class Collective {
public:
    // nccl_id: the 128-byte ncclUniqueId created by rank 0 and shared by the
    // caller (e.g. over torch.distributed); every rank of the group calls this.
    Collective(const void* nccl_id, int rank, int size);
    ~Collective();
    Collective(const Collective&) = delete;
    Collective& operator=(const Collective&) = delete;
    // In-place sum over the group of n floats on `stream`.
    void allreduce_sum(float* data, std::size_t n, cudaStream_t stream);
    // recv[r * bytes .. (r + 1) * bytes) = rank r's `bytes` of send, on every rank.
    void allgather(const void* send, void* recv, std::size_t bytes, cudaStream_t stream);
    int rank() const { return rank_; }
    int size() const { return size_; }

private:
    void* lib_ = nullptr;
    void* comm_ = nullptr;
    int rank_ = 0, size_ = 1;
};

}  // namespace tvara
