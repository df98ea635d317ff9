// tvara_paged_attention_noalloc: the paged attention of tvara_paged_attention
// run on a scratch area that lives in this library's own device code (a
// file-scope __device__ array) instead of caller-provided device memory.
//
// It serves callers that cannot allocate device memory at the point of the
// call: hosts binding the C ABI through an FFI with no device allocator of
// their own, code whose device memory is entirely owned by another
// framework's caching allocator, and code that must not pay cudaMalloc's
// implicit device-wide synchronisation between launches.  Nothing here calls
// cudaMalloc, cudaFree or any allocating library routine.
//
// Limits and rules (also stated in include/tvara_kernels.h):
//  * the scratch holds kScratchBytes; arguments whose scratch requirement
//    (tvara_paged_attention_workspace) exceeds it are rejected with an error
//    before any device work is enqueued;
//  * the first call on a device, with that device current, resolves the
//    scratch address (cudaGetSymbolAddress, which may load this library's
//    device code onto the device);
//  * like tvara_paged_attention, a call stages its block tables and work list
//    from a host buffer and waits for the kernels' error word before it
//    returns, so it is synchronous on `stream` and cannot be recorded into a
//    CUDA graph (a capturing stream is refused before anything is enqueued);
//  * there is one scratch per device: calls that overlap on one device (two
//    streams, or two host threads, before the first has finished on the
//    device) race on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/tvara_kernels.h"

namespace tvara {
std::string& last_error();
}

namespace {

constexpr std::size_t kScratchBytes = std::size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

// Block tables, split-KV work list, partial results and the error word of one
// call.  Only the error word must start at zero: tvara_paged_attention clears
// it on the stream before every launch and writes everything else before it
// is read.
static __device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch[kMaxDevices] = {};

// Resolves (once per device, with that device current) the scratch address.
void* scratch_for_current_device() {
    int device = -1;
    cudaError_t rc = cudaGetDevice(&device);
    if (rc != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice failed: ") + cudaGetErrorString(rc));
    if (device < 0 || device >= kMaxDevices) throw std::runtime_error("device ordinal out of range for static scratch");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch[device]) {
        void* p = nullptr;
        rc = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (rc != cudaSuccess || !p)
            throw std::runtime_error(std::string("cannot resolve static attention scratch: ") + cudaGetErrorString(rc));
        g_scratch[device] = p;
    }
    return g_scratch[device];
}

}  // namespace

extern "C" {

size_t tvara_paged_attention_noalloc_max(void) { return kScratchBytes; }

int tvara_paged_attention_noalloc(const tvara_attention_args* args, void* stream) {
    const std::size_t need = tvara_paged_attention_workspace(args);
    if (!need) return -1;  // invalid arguments: the error text is already set
    if (need > kScratchBytes) {
        tvara::last_error() = "paged attention scratch of " + std::to_string(need) +
                              " bytes exceeds the static maximum of " + std::to_string(kScratchBytes) + " bytes";
        return -1;
    }
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &capturing) != cudaSuccess ||
        capturing != cudaStreamCaptureStatusNone) {
        tvara::last_error() = "paged attention cannot be captured into a CUDA graph";
        return -1;
    }
    void* scratch = nullptr;
    try {
        scratch = scratch_for_current_device();
    } catch (const std::exception& e) {
        tvara::last_error() = e.what();
        return -1;
    }
    return tvara_paged_attention(args, scratch, kScratchBytes, stream);
}

}  // extern "C"
