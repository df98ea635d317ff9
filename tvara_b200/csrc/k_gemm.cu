// Projection dispatch: the CUDA-core GEMV streams weights once per group of
// at most four tokens; larger token counts go to the tensor-core kernel when
// it supports the matrix.
#include "kernels.cuh"

namespace tvara {

bool gemm_tc_supported(const DeviceMatrix&, int) { return false; }

void launch_gemm_tc(const GemmArgs&, void*, std::size_t, cudaStream_t) {
    throw std::logic_error("tensor-core projection not available for this matrix");
}

std::size_t gemm_tc_workspace(int, int) { return 0; }

void launch_projection(const GemmArgs& a, void* workspace, std::size_t workspace_bytes, cudaStream_t s) {
    if (gemm_tc_supported(a.w, a.tokens)) launch_gemm_tc(a, workspace, workspace_bytes, s);
    else launch_gemv(a, s);
}

}  // namespace tvara
