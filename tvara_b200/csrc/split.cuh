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

}  // namespace tvara
