// Tensor Memory Accelerator helpers shared by the kernels: the driver's
// tensor-map encoder (resolved once through the runtime) and the 2-D tiled
// global -> shared copy completing on an mbarrier.  Every map built here is
// over this GPU's own memory and every copy is issued per CTA.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>
#include <stdexcept>

namespace tvara {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// Copies the box at element coordinates (x, y) of `map` to `dst` (shared
// memory), completing `bytes` of transaction count on the mbarrier `bar`.
// x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(unsigned dst, const CUtensorMap* map, int x, int y, unsigned bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

}  // namespace tvara
