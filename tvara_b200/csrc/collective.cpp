// NCCL over NVLink/NVSwitch for the tensor-parallel allreduce after o_proj and
// down_proj and the gathers of the vocabulary-split LM head.  Only the stable
// NCCL C entry points are used.
#include "collective.hpp"

#include <dlfcn.h>

#include <cstring>
#include <stdexcept>
#include <string>

namespace tvara {
namespace {

struct UniqueId {
    char internal[128];
};
using InitRank = int (*)(void**, int, UniqueId, int);
using AllReduce = int (*)(const void*, void*, std::size_t, int, int, void*, cudaStream_t);
using AllGather = int (*)(const void*, void*, std::size_t, int, void*, cudaStream_t);
using Destroy = int (*)(void*);
using ErrorString = const char* (*)(int);
constexpr int kNcclFloat32 = 7;
constexpr int kNcclUint8 = 1;
constexpr int kNcclSum = 0;

void* open_nccl() {
    for (const char* name : {"libnccl.so.2", "libnccl.so"}) {
        if (void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL)) return h;
    }
    throw std::runtime_error("tensor parallelism needs libnccl.so.2 (not found)");
}

template <class F>
F sym(void* lib, const char* name) {
    auto f = reinterpret_cast<F>(dlsym(lib, name));
    if (!f) throw std::runtime_error(std::string("NCCL symbol missing: ") + name);
    return f;
}

void check(void* lib, int code, const char* what) {
    if (code != 0) {
        const char* msg = sym<ErrorString>(lib, "ncclGetErrorString")(code);
        throw std::runtime_error(std::string(what) + ": " + (msg ? msg : "NCCL error"));
    }
}

}  // namespace

Collective::Collective(const void* nccl_id, int rank, int size) : rank_(rank), size_(size) {
    lib_ = open_nccl();
    UniqueId id;
    std::memcpy(id.internal, nccl_id, sizeof(id.internal));
    check(lib_, sym<InitRank>(lib_, "ncclCommInitRank")(&comm_, size, id, rank), "ncclCommInitRank");
}

Collective::~Collective() {
    if (comm_ && lib_) sym<Destroy>(lib_, "ncclCommDestroy")(comm_);
}

void Collective::allreduce_sum(float* data, std::size_t n, cudaStream_t stream) {
    check(lib_, sym<AllReduce>(lib_, "ncclAllReduce")(data, data, n, kNcclFloat32, kNcclSum, comm_, stream),
          "ncclAllReduce");
}

void Collective::allgather(const void* send, void* recv, std::size_t bytes, cudaStream_t stream) {
    check(lib_, sym<AllGather>(lib_, "ncclAllGather")(send, recv, bytes, kNcclUint8, comm_, stream), "ncclAllGather");
}

}  // namespace tvara
