// Shared host/device definitions for the B200 decode/prefill engine.
#pragma once
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace tvara {

// GGUF storage types on this path (reference gguf.hpp:152-170).
enum TensorType : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12 };

inline bool block_shape(int type, std::size_t& elems, std::size_t& bytes) {
    switch (type) {
        case kF32: elems = 1; bytes = 4; return true;
        case kF16: elems = 1; bytes = 2; return true;
        case kQ4_0: elems = 32; bytes = 18; return true;
        case kQ8_0: elems = 32; bytes = 34; return true;
        case kQ4_K: elems = 256; bytes = 144; return true;
        default: return false;
    }
}

// A weight matrix [rows][cols] resident in HBM in the engine's split layout:
//   qs   -- per row, the quantised codes (F32/F16: the values)
//            Q8_0: int8 [cols]; Q4_0: 16 B per 32 (GGUF nibble order);
//            Q4_K: 128 B per 256 (GGUF nibble order); F16: half; F32: float
//   meta -- per row, the block headers: Q8_0/Q4_0 fp16 d per 32; Q4_K the
//            16-byte {d, dmin, scales[12]} per 256; none for F32/F16.
// Splitting headers from codes keeps every row 16-byte aligned so kernels
// stream it with 128-bit loads; the arithmetic is unchanged.
struct DeviceMatrix {
    int type = kF32;
    int rows = 0, cols = 0;
    const std::uint8_t* qs = nullptr;
    const std::uint8_t* meta = nullptr;
    std::size_t qs_row = 0;    // bytes per row in qs
    std::size_t meta_row = 0;  // bytes per row in meta
    // Per row, the power of two (2^shift) that brings the row's largest
    // |value| into [2^14, 2^15): the tensor-core path scales by it before the
    // exact hi+lo FP16 split.  Null until computed (then only GEMV is used).
    const signed char* row_shift = nullptr;
    // Optional exact FP16 planes of the scaled values (value * 2^row_shift =
    // hi + lo), [rows][cols] each: the tensor-core path then streams them by
    // TMA instead of dequantising the packed rows.  Null when not built.
    const std::uint16_t* plane_hi = nullptr;
    const std::uint16_t* plane_lo = nullptr;
    // Optional Q4_K tensor-core form (instead of the planes above): a Q4_K
    // value is d*sc*q - dmin*m per 32-element sub-block, and sc*q is an
    // integer below 1024, exact in FP16.  qplane [rows][cols] FP16 holds sc*q;
    // qscale [rows][cols/256] the block scales d; qmin_hi / qmin_lo
    // [rows][cols/32] FP16 the exact split of dmin*m * 2^qmin_shift[row].
    const std::uint16_t* qplane = nullptr;
    // Packed form (qplane null): the same factorisation with the codes read
    // from the packed rows (qs) and sc*q built in shared memory by the
    // kernel; qsc [rows][cols/32] holds each sub-block's 6-bit scale sc.
    const std::uint8_t* qsc = nullptr;
    const float* qscale = nullptr;
    const std::uint16_t* qmin_hi = nullptr;
    const std::uint16_t* qmin_lo = nullptr;
    const signed char* qmin_shift = nullptr;
};

inline std::size_t qs_row_bytes(int type, std::size_t cols) {
    switch (type) {
        case kF32: return cols * 4;
        case kF16: return cols * 2;
        case kQ8_0: return cols;
        case kQ4_0: return cols / 2;
        case kQ4_K: return cols / 2;
    }
    return 0;
}
inline std::size_t meta_row_bytes(int type, std::size_t cols) {
    switch (type) {
        case kQ8_0:
        case kQ4_0: return cols / 32 * 2;
        case kQ4_K: return cols / 256 * 16;
    }
    return 0;
}

class CudaError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

// Kernel launches issued by this library since load (all handles, all
// threads); every launch wrapper adds its launches.
void note_launches(unsigned long long n = 1);
unsigned long long launches();

}  // namespace tvara

// After a kernel launch: count it and surface launch errors.
#define TVARA_LAUNCHED()                          \
    do {                                          \
        ::tvara::note_launches();                 \
        TVARA_CUDA(cudaGetLastError());           \
    } while (0)

#define TVARA_CUDA(call)                                                                      \
    do {                                                                                      \
        cudaError_t err__ = (call);                                                           \
        if (err__ != cudaSuccess)                                                             \
            throw ::tvara::CudaError(std::string("CUDA error: ") + cudaGetErrorString(err__) + \
                                     " at " + __FILE__ + ":" + std::to_string(__LINE__));     \
    } while (0)
