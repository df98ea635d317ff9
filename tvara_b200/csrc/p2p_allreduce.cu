// Two-shot allreduce of the tensor-parallel residual over NVLink peer memory.
//
// After o_proj and down_proj every rank holds a partial of the residual
// [T][hidden] in the same buffer of its step scratch (x_, identical offsets
// on every rank).  One kernel per allreduce:
//   1. barrier: block 0 tells every rank this rank's partial is in place (one
//      system-scope release add into each rank's arrival counter); every CTA
//      waits until its own counter shows all ranks;
//   2. reduce-scatter + all-gather in one pass: rank k owns the k-th slice of
//      the elements; its threads load their elements of that slice from every
//      rank's buffer (peer loads over NVLink, U elements per rank in flight per
//      thread), add the partials in rank order 0..size-1 (so every rank ends
//      with bit-identical sums) and store the sum into every rank's buffer
//      (peer stores);
//   3. barrier: each CTA, after its stores and a system-scope fence, counts
//      itself on a local counter; the CTA that completes the count tells every
//      rank that this rank's stores are done and waits until all ranks have
//      told it the same, so the kernel ends only once every peer has finished
//      writing this rank's buffer and the next kernel on the stream reads a
//      complete sum.  (A peer's stores into this rank's buffer follow its loads
//      of this rank's partial, so they also mark the end of those reads.)
// Per rank the traffic is 2 (size-1)/size of the buffer each way -- the
// two-shot minimum -- in one launch and without staging copies.  Buffers are
// shared once at set-up through CUDA IPC handles exchanged with an NCCL
// all-gather.  Counters only grow; the host keeps the cumulative value each
// wait expects (the grid, and so the CTA count, varies with the size), so
// nothing is reset between calls and wrap-around is harmless.  Every wait is
// bounded: after the limit the kernel records error 5 and returns instead of
// spinning on.  Only plain loads, stores and atomics reach peer memory (no
// multicast).
#include "p2p_allreduce.hpp"

#include <algorithm>
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
    unsigned* counters[kMaxPeerRanks];   // every rank's counters: [0] arrivals, [1] ranks done, [2] local CTAs done
    int rank, size;
    long long slice4;                    // float4 elements per rank slice
    unsigned arrive_target;              // cumulative counters[rank][0] this call waits for
    unsigned done_target;                // cumulative counters[rank][1] this call waits for
    unsigned cta_target;                 // cumulative counters[rank][2] once every CTA of this call counted
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
// Waits (bounded) until *counter has reached target (modulo 2^32); false on
// timeout (error recorded).
__device__ bool wait_count(const unsigned* counter, unsigned target, int* err) {
    for (unsigned i = 0; i < kPeerSpin; ++i) {
        if (int(ld_acquire_sys(counter) - target) >= 0) return true;
        if (i > 16) __nanosleep(128);
    }
    atomicExch(err, 5);
    return false;
}

__device__ __forceinline__ void add4(float4& s, const float4& v) {
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
}

// R ranks; U slice elements per thread per pass, each loaded from every rank
// before any is summed (U * R float4 loads in flight).
template <int R, int U>
__global__ void __launch_bounds__(kReduceThreads) p2p_allreduce_kernel(PeerArgs a) {
    __shared__ int ok, last;
    // 1. partials in place everywhere
    if (blockIdx.x == 0 && threadIdx.x < a.size) red_release_sys(a.counters[threadIdx.x], 1u);
    if (threadIdx.x == 0) ok = wait_count(a.counters[a.rank], a.arrive_target, a.err);
    __syncthreads();
    if (ok) {
        // 2. this rank's slice: sum in rank order, store everywhere
        const long long begin = a.rank * a.slice4, end = begin + a.slice4;
        const long long stride = (long long)gridDim.x * blockDim.x;
        for (long long i0 = begin + blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < end; i0 += U * stride) {
            float4 v[R][U];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const long long i = i0 + u * stride;
                    v[r][u] = i < end ? a.buf[r][i] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const long long i = i0 + u * stride;
                if (i >= end) break;
                float4 s = v[0][u];
#pragma unroll
                for (int r = 1; r < R; ++r) add4(s, v[r][u]);
#pragma unroll
                for (int r = 0; r < R; ++r) a.buf[r][i] = s;
            }
        }
    }
    // 3. this CTA's stores are out; the last CTA of the rank tells every rank
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(a.counters[a.rank] + 2, 1u) == a.cta_target - 1u;
    }
    __syncthreads();
    if (last) {
        if (threadIdx.x == 0) __threadfence_system();
        __syncwarp();
        if (threadIdx.x < a.size) red_release_sys(a.counters[threadIdx.x] + 1, 1u);
        if (threadIdx.x == 0 && ok) wait_count(a.counters[a.rank] + 1, a.done_target, a.err);
    }
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
    a.err = err;
    // U * size float4 loads in flight per thread: about 8 for any group size
    const int U = size_ <= 2 ? 4 : size_ <= 4 ? 2 : 1;
    const long long per_cta = (long long)kReduceThreads * U;
    const int grid = int(std::max<long long>(1, std::min<long long>(sms_, (a.slice4 + per_cta - 1) / per_cta)));
    arrived_ += unsigned(size_);
    done_ += unsigned(size_);
    ctas_ += unsigned(grid);
    a.arrive_target = arrived_;
    a.done_target = done_;
    a.cta_target = ctas_;
    switch (size_) {
        case 2: p2p_allreduce_kernel<2, 4><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 3: p2p_allreduce_kernel<3, 2><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 4: p2p_allreduce_kernel<4, 2><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 5: p2p_allreduce_kernel<5, 1><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 6: p2p_allreduce_kernel<6, 1><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 7: p2p_allreduce_kernel<7, 1><<<grid, kReduceThreads, 0, stream>>>(a); break;
        case 8: p2p_allreduce_kernel<8, 1><<<grid, kReduceThreads, 0, stream>>>(a); break;
        default: throw std::invalid_argument("peer allreduce needs 2 to 8 ranks");
    }
    TVARA_LAUNCHED();
}

}  // namespace tvara
