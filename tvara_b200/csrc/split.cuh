// Exact two-part FP16 split used by the tensor-core projection.
#pragma once

#include <cuda_fp16.h>

namespace tvara {

// Values already scaled to |x| < 2^15 (per weight row / per token by a power
// of two): hi is x rounded to a multiple of 16 (adding and removing
// 1.5 * 2^27, whose ulp is 16), which FP16 holds exactly; lo = x - hi lies in
// [-8, 8] and rounds to FP16 with an error of at most 2^-9 -- the same
// absolute bound as a round-to-nearest hi, without converting FP16 back to
// F32.  hi + lo carries x to ~2^-24 of the row / token maximum.
__device__ __forceinline__ void split_exact(float x0, float x1, unsigned& hi, unsigned& lo) {
    constexpr float kRound16 = 201326592.f;  // 1.5 * 2^27
    const float h0 = __fsub_rn(__fadd_rn(x0, kRound16), kRound16);
    const float h1 = __fsub_rn(__fadd_rn(x1, kRound16), kRound16);
    const __half2 h = __floats2half2_rn(h0, h1);
    const __half2 l = __floats2half2_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
    hi = *reinterpret_cast<const unsigned*>(&h);
    lo = *reinterpret_cast<const unsigned*>(&l);
}

// The Q4_K min term's B operand, written by the kernels that split a token's
// activations: when lanes 8m..8m+7 hold the eight float4s of one 32-element
// sub-block (float4 k at lane k % 32), the sub-block sum scaled by
// 2^(shift - 5) (below 2^15 since every |x * 2^shift| is) is split exactly
// into shi / slo [unit].  Every lane of the warp calls it (shuffles).
__device__ __forceinline__ void subblock_sum_split(float4 v, int k, bool valid, float f32, __half* shi, __half* slo) {
    float sum = valid ? (v.x + v.y) + (v.z + v.w) : 0.f;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (valid && (k & 7) == 0) {
        unsigned hi, lo;
        split_exact(sum * f32, 0.f, hi, lo);
        shi[k >> 3] = __ushort_as_half((unsigned short)(hi & 0xffffu));
        slo[k >> 3] = __ushort_as_half((unsigned short)(lo & 0xffffu));
    }
}

}  // namespace tvara
