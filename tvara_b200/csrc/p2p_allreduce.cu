// Two-shot allreduce of the tensor-parallel residual over NVLink peer memory.
//
// After o_proj and down_proj every rank holds a partial of the residual
// [T][hidden] in the same buffer of its step scratch (x_, identical offsets
// on every rank).  One kernel per allreduce:
//   1. barrier: each rank tells every rank its partial is in place (one
//      system-scope atomic add into each rank's counter) and waits for all;
//   2. reduce-scatter + all-gather in one pass: rank k owns the k-th slice of
//      the elements; its CTAs read that slice from every rank's buffer (peer
//      loads over NVLink), add the partials in rank order 0..size-1 (so every
//      rank ends with bit-identical sums) and store the sum into every rank's
//      buffer (peer stores);
//   3. barrier: each CTA, after a system-scope fence, counts itself into every
//      rank's second counter; a rank's CTAs leave once all ranks' CTAs have,
//      so the next kernel on each stream reads a complete sum.
// Per rank the traffic is 2 (size-1)/size of the buffer each way -- the
// two-shot minimum -- in one launch and without staging copies.  Buffers are
// shared once at set-up through CUDA IPC handles exchanged with an NCCL
// all-gather.  Counters only grow (epoch e waits for e * size and e * size *
// CTAs), so nothing is reset between calls.  Every wait is bounded: after
// the limit the kernel records error 5 and returns instead of spinning on.
// Only plain loads, stores and atomics reach peer memory (no multicast).
#include "p2p_allreduce.hpp"

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace tvara {
namespace {

constexpr unsigned kPeerSpin = 1u << 24;
constexpr int kReduceThreads = 512;

struct PeerArgs {
    float4* buf[kMaxPeerRanks];          // every rank's buffer (this rank's own included)
    unsigned* counters[kMaxPeerRanks];   // every rank's two counters
    int rank, size;
    long long slice4;                    // float4 elements per rank slice
    unsigned epoch;
    int* err;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Waits (bounded) until *counter >= target; false on timeout (error recorded).
__device__ bool wait_count(const unsigned* counter, unsigned target, int* err) {
    for (unsigned i = 0; i < kPeerSpin; ++i) {
        if (int(ld_acquire_sys(counter) - target) >= 0) return true;
        if (i > 16) __nanosleep(128);
    }
    atomicExch(err, 5);
    return false;
}

__global__ void __launch_bounds__(kReduceThreads) p2p_allreduce_kernel(PeerArgs a) {
    __shared__ int ok;
    // 1. partials in place everywhere
    if (blockIdx.x == 0 && threadIdx.x < a.size) red_release_sys(a.counters[threadIdx.x], 1u);
    if (threadIdx.x == 0) ok = wait_count(a.counters[a.rank], a.epoch * unsigned(a.size), a.err);
    __syncthreads();
    if (ok) {
        // 2. this rank's slice: sum in rank order, store everywhere
        const long long begin = a.rank * a.slice4, end = begin + a.slice4;
        for (long long i = begin + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < end;
             i += (long long)gridDim.x * blockDim.x) {
            float4 s = a.buf[0][i];
            for (int r = 1; r < a.size; ++r) {
                const float4 v = a.buf[r][i];
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            for (int r = 0; r < a.size; ++r) a.buf[r][i] = s;
        }
    }
    // 3. every CTA of every rank done storing
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.size) red_release_sys(a.counters[threadIdx.x] + 1, 1u);
    if (threadIdx.x == 0 && ok) wait_count(a.counters[a.rank] + 1, a.epoch * unsigned(a.size) * gridDim.x, a.err);
    __syncthreads();
}

}  // namespace

PeerAllreduce::PeerAllreduce(Collective& coll, float* buffer, std::size_t capacity, cudaStream_t stream)
    : rank_(coll.rank()), size_(coll.size()), capacity_(capacity) {
    if (size_ > kMaxPeerRanks) throw std::invalid_argument("peer allreduce supports at most 8 ranks");
    int dev = 0;
    TVARA_CUDA(cudaGetDevice(&dev));
    TVARA_CUDA(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, dev));
    TVARA_CUDA(cudaMalloc(&counters_, 256));
    TVARA_CUDA(cudaMemset(counters_, 0, 256));
    // this rank's two IPC handles, gathered from every rank over NCCL
    struct Handles {
        cudaIpcMemHandle_t buf, counters;
    } mine{};
    TVARA_CUDA(cudaIpcGetMemHandle(&mine.buf, buffer));
    TVARA_CUDA(cudaIpcGetMemHandle(&mine.counters, counters_));
    void* dev_handles = nullptr;
    TVARA_CUDA(cudaMalloc(&dev_handles, sizeof(Handles) * (size_ + 1)));
    std::vector<Handles> all(size_);
    try {
        TVARA_CUDA(cudaMemcpyAsync(static_cast<char*>(dev_handles) + sizeof(Handles) * size_, &mine, sizeof(Handles),
                                   cudaMemcpyHostToDevice, stream));
        coll.allgather(static_cast<char*>(dev_handles) + sizeof(Handles) * size_, dev_handles, sizeof(Handles), stream);
        TVARA_CUDA(cudaMemcpyAsync(all.data(), dev_handles, sizeof(Handles) * size_, cudaMemcpyDeviceToHost, stream));
        TVARA_CUDA(cudaStreamSynchronize(stream));
    } catch (...) {
        cudaFree(dev_handles);
        throw;
    }
    cudaFree(dev_handles);
    for (int r = 0; r < size_; ++r) {
        if (r == rank_) {
            bufs_[r] = buffer;
            cnts_[r] = counters_;
            continue;
        }
        void* b = nullptr;
        void* c = nullptr;
        TVARA_CUDA(cudaIpcOpenMemHandle(&b, all[r].buf, cudaIpcMemLazyEnablePeerAccess));
        opened_.push_back(b);
        TVARA_CUDA(cudaIpcOpenMemHandle(&c, all[r].counters, cudaIpcMemLazyEnablePeerAccess));
        opened_.push_back(c);
        bufs_[r] = static_cast<float*>(b);
        cnts_[r] = static_cast<unsigned*>(c);
    }
}

PeerAllreduce::~PeerAllreduce() {
    for (void* p : opened_) cudaIpcCloseMemHandle(p);
    if (counters_) cudaFree(counters_);
}

bool PeerAllreduce::applies(const float* data, std::size_t n) const {
    return data == bufs_[rank_] && n <= capacity_ && n % (4 * std::size_t(size_)) == 0 && n > 0;
}

void PeerAllreduce::allreduce_sum(float* data, std::size_t n, int* err, cudaStream_t stream) {
    if (!applies(data, n)) throw std::invalid_argument("peer allreduce: buffer or size not registered");
    PeerArgs a{};
    for (int r = 0; r < size_; ++r) {
        a.buf[r] = reinterpret_cast<float4*>(bufs_[r]);
        a.counters[r] = cnts_[r];
    }
    a.rank = rank_;
    a.size = size_;
    a.slice4 = (long long)(n / 4 / size_);
    a.epoch = ++epoch_;
    a.err = err;
    const long long per_cta = (long long)kReduceThreads * 2;
    const int grid = int(std::max<long long>(1, std::min<long long>(sms_, (a.slice4 + per_cta - 1) / per_cta)));
    // the grid must be the same on every rank (it sets the second barrier's count): it depends on n only
    p2p_allreduce_kernel<<<grid, kReduceThreads, 0, stream>>>(a);
    TVARA_LAUNCHED();
}

}  // namespace tvara
