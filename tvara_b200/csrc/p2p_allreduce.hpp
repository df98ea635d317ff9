// Peer-memory allreduce for a tensor-parallel group whose ranks are GPUs of
// one NVLink/NVSwitch domain (p2p_allreduce.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

#include "collective.hpp"
#include "common.hpp"

namespace tvara {

constexpr int kMaxPeerRanks = 8;

class PeerAllreduce {
public:
    // `buffer`: the start of a cudaMalloc allocation holding up to `capacity`
    // floats at the same offset on every rank; every rank of `coll` calls
    // this collectively (it all-gathers the IPC handles).
    PeerAllreduce(Collective& coll, float* buffer, std::size_t capacity, cudaStream_t stream);
    ~PeerAllreduce();
    PeerAllreduce(const PeerAllreduce&) = delete;
    PeerAllreduce& operator=(const PeerAllreduce&) = delete;
    // Whether allreduce_sum takes (data, n): the registered buffer, a size that
    // splits into float4 slices per rank, within capacity.
    bool applies(const float* data, std::size_t n) const;
    // In-place sum over the group on `stream`; err receives 5 if a peer never
    // arrived within the wait limit.  Every rank calls it in the same order.
    void allreduce_sum(float* data, std::size_t n, int* err, cudaStream_t stream);

private:
    int rank_ = 0, size_ = 1, sms_ = 148;
    std::size_t capacity_ = 0;
    // cumulative values this rank's counters reach once the last call issued
    // completes: arrivals, ranks done, this rank's CTAs done
    unsigned arrived_ = 0, done_ = 0, ctas_ = 0;
    unsigned* counters_ = nullptr;  // this rank's three barrier counters
    float* bufs_[kMaxPeerRanks] = {};
    unsigned* cnts_[kMaxPeerRanks] = {};
    std::vector<void*> opened_;
};

}  // namespace tvara
