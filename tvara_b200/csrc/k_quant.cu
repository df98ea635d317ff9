// Quantised block unpack, repack and the CUDA-core projection (decode GEMV).
//
// Device layout of a projection (see DeviceMatrix): qs streams the codes of
// each row, meta the block headers.  Q4_K codes are regrouped at load so a
// 16-byte unit holds one 32-element sub-block in Q4_0's nibble order (byte j:
// element j low, element j+16 high); the value of every element is still
// d*sc*q - dmin*m of reference core/include/tvara/quant.hpp:70-84.
#include <cstdint>

#include "kernels.cuh"
#include "split.cuh"

namespace tvara {
namespace {

constexpr int kWarps = 4;  // warps per CTA of the GEMV (small CTAs: the whole grid is resident at once)

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Reference half_to_float (quant.hpp:14-29) in integer arithmetic, so NaN
// payloads and subnormals come out bit-identical.
__device__ __forceinline__ float half_bits_to_float(unsigned h) {
    const unsigned sign = (h & 0x8000u) << 16;
    unsigned e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 0) {
        if (!m) {
            bits = sign;
        } else {
            int ex = -14;
            while ((m & 1024u) == 0) {
                m <<= 1;
                --ex;
            }
            bits = sign | (unsigned(ex + 127) << 23) | ((m & 1023u) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ float h2f(unsigned short h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ void q4k_scale_min(const unsigned char* s, int g, unsigned& sc, unsigned& m) {
    if (g < 4) {
        sc = s[g] & 63u;
        m = s[g + 4] & 63u;
    } else {
        sc = (s[g + 4] & 15u) | ((unsigned)(s[g - 4] >> 6) << 4);
        m = (s[g + 4] >> 4) | ((unsigned)(s[g] >> 6) << 4);
    }
}
// Same decode from the 12 scale bytes held in three words.
// Branch-free (g differs between the lanes of a warp): with k = g & 3 and
// the k-th bytes y, z, w of the three scale words, sub-blocks 0-3 take
// (y & 63, z & 63) and 4-7 take (w & 15 | (y >> 6) << 4, w >> 4 | (z >> 6) << 4).
__device__ __forceinline__ void q4k_scale_min_w(unsigned w0, unsigned w1, unsigned w2, int g, float& sc, float& m) {
    const unsigned sh = 8u * unsigned(g & 3);
    const unsigned y = (w0 >> sh) & 255u, z = (w1 >> sh) & 255u, w = (w2 >> sh) & 255u;
    const bool low = g < 4;
    const unsigned s = low ? (y & 63u) : ((w & 15u) | ((y >> 6) << 4));
    const unsigned mm = low ? (z & 63u) : ((w >> 4) | ((z >> 6) << 4));
    sc = float(s);
    m = float(mm);
}

// ------------------------------------------------------------------ unpack
// The reference is built for x86-64, where SSE arithmetic returns the first
// NaN operand (quieted) and an invalid operation (inf*0, inf-inf) returns the
// negative default NaN 0xFFC00000; the GPU returns a canonical NaN instead.
// For bit-identical unpacking of blocks whose scales are NaN or inf, the
// unpack kernel applies the x86 rule; finite results are plain IEEE _rn ops.
__device__ __forceinline__ float x86_nan(float a) { return __uint_as_float(__float_as_uint(a) | 0x00400000u); }
__device__ __forceinline__ float x86_mul(float a, float b) {
    if (isnan(a)) return x86_nan(a);
    if (isnan(b)) return x86_nan(b);
    const float r = __fmul_rn(a, b);
    return isnan(r) ? __uint_as_float(0xFFC00000u) : r;
}
__device__ __forceinline__ float x86_sub(float a, float b) {
    if (isnan(a)) return x86_nan(a);
    if (isnan(b)) return x86_nan(b);
    const float r = __fsub_rn(a, b);
    return isnan(r) ? __uint_as_float(0xFFC00000u) : r;
}

// One thread per output element; arithmetic and rounding order as the
// reference dequantisers (no contraction).
__global__ void dequant_kernel(int type, const unsigned char* src, std::size_t nblocks, float* out) {
    const std::size_t per = type == kQ4_K ? 256 : (type == kQ8_0 || type == kQ4_0) ? 32 : 1;
    const std::size_t total = nblocks * per;
    for (std::size_t i = blockIdx.x * std::size_t(blockDim.x) + threadIdx.x; i < total;
         i += std::size_t(gridDim.x) * blockDim.x) {
        const std::size_t b = i / per, e = i % per;
        float v;
        if (type == kF32) {
            v = __uint_as_float(src[4 * b] | (src[4 * b + 1] << 8) | (src[4 * b + 2] << 16) | (unsigned(src[4 * b + 3]) << 24));
        } else if (type == kF16) {
            v = half_bits_to_float(src[2 * b] | (src[2 * b + 1] << 8));
        } else if (type == kQ8_0) {
            const unsigned char* blk = src + b * 34;
            v = x86_mul(half_bits_to_float(blk[0] | (blk[1] << 8)), float((signed char)blk[2 + e]));
        } else if (type == kQ4_0) {
            const unsigned char* blk = src + b * 18;
            const unsigned q = e < 16 ? (blk[2 + e] & 15u) : (blk[2 + e - 16] >> 4);
            v = x86_mul(half_bits_to_float(blk[0] | (blk[1] << 8)), float(int(q) - 8));
        } else {  // Q4_K
            const unsigned char* blk = src + b * 144;
            const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
            const float dmin = half_bits_to_float(blk[2] | (blk[3] << 8));
            const int g = int(e / 32), j = int(e % 32);
            unsigned sc, m;
            q4k_scale_min(blk + 4, g, sc, m);
            const unsigned packed = blk[16 + (g / 2) * 32 + j];
            const unsigned q = (g % 2) ? (packed >> 4) : (packed & 15u);
            v = x86_sub(x86_mul(x86_mul(d, float(sc)), float(q)), x86_mul(dmin, float(m)));
        }
        out[i] = v;
    }
}

// GGUF rows -> (qs, meta).  One thread per output block.
__global__ void repack_kernel(int type, const unsigned char* src, int rows, int cols, unsigned char* qs,
                              unsigned char* meta) {
    const int per = type == kQ4_K ? 256 : 32;
    const int nb = cols / per;
    const std::size_t in_row = std::size_t(nb) * (type == kQ4_K ? 144 : type == kQ8_0 ? 34 : 18);
    const std::size_t total = std::size_t(rows) * nb;
    for (std::size_t i = blockIdx.x * std::size_t(blockDim.x) + threadIdx.x; i < total;
         i += std::size_t(gridDim.x) * blockDim.x) {
        const std::size_t r = i / nb, b = i % nb;
        if (type == kQ8_0) {
            const unsigned char* blk = src + r * in_row + b * 34;
            unsigned char* q = qs + r * std::size_t(cols) + b * 32;
            for (int j = 0; j < 32; ++j) q[j] = blk[2 + j];
            meta[(r * nb + b) * 2] = blk[0];
            meta[(r * nb + b) * 2 + 1] = blk[1];
        } else if (type == kQ4_0) {
            const unsigned char* blk = src + r * in_row + b * 18;
            unsigned char* q = qs + r * std::size_t(cols / 2) + b * 16;
            for (int j = 0; j < 16; ++j) q[j] = blk[2 + j];
            meta[(r * nb + b) * 2] = blk[0];
            meta[(r * nb + b) * 2 + 1] = blk[1];
        } else {  // Q4_K: regroup each 32-element sub-block into one 16-byte unit
            const unsigned char* blk = src + r * in_row + b * 144;
            unsigned char* q = qs + r * std::size_t(cols / 2) + b * 128;
            for (int g = 0; g < 8; ++g)
                for (int j = 0; j < 16; ++j) {
                    const unsigned lo = g % 2 ? blk[16 + (g / 2) * 32 + j] >> 4 : blk[16 + (g / 2) * 32 + j] & 15u;
                    const unsigned hi =
                        g % 2 ? blk[16 + (g / 2) * 32 + j + 16] >> 4 : blk[16 + (g / 2) * 32 + j + 16] & 15u;
                    q[g * 16 + j] = (unsigned char)(lo | (hi << 4));
                }
            for (int j = 0; j < 16; ++j) meta[(r * nb + b) * 16 + j] = blk[j];
        }
    }
}

// Value of element k of row r in the engine layout (embedding gather and
// the finite check).  Same operation order as the reference dequantisers.
__device__ __forceinline__ float element(const DeviceMatrix& w, long long r, int k) {
    const unsigned char* qs = w.qs + r * w.qs_row;
    const unsigned char* meta = w.meta + r * w.meta_row;
    switch (w.type) {
        case kF32: return reinterpret_cast<const float*>(qs)[k];
        case kF16: return h2f(reinterpret_cast<const unsigned short*>(qs)[k]);
        case kQ8_0: {
            const unsigned short d = reinterpret_cast<const unsigned short*>(meta)[k / 32];
            return __fmul_rn(half_bits_to_float(d), float((signed char)qs[k]));
        }
        case kQ4_0: {
            const unsigned short d = reinterpret_cast<const unsigned short*>(meta)[k / 32];
            const unsigned char byte = qs[(k / 32) * 16 + (k % 16)];
            const unsigned q = (k % 32) < 16 ? (byte & 15u) : (byte >> 4);
            return __fmul_rn(half_bits_to_float(d), float(int(q) - 8));
        }
        default: {  // Q4_K
            const int b = k / 256, g = (k % 256) / 32, j = k % 32;
            const unsigned char* m = meta + b * 16;
            const float d = half_bits_to_float(m[0] | (m[1] << 8));
            const float dmin = half_bits_to_float(m[2] | (m[3] << 8));
            unsigned sc, mn;
            q4k_scale_min(m + 4, g, sc, mn);
            const unsigned char byte = qs[(k / 32) * 16 + (j % 16)];
            const unsigned q = j < 16 ? (byte & 15u) : (byte >> 4);
            return __fsub_rn(__fmul_rn(__fmul_rn(d, float(sc)), float(q)), __fmul_rn(dmin, float(mn)));
        }
    }
}

__global__ void finite_kernel(DeviceMatrix w, int* flag) {
    const long long total = (long long)w.rows * w.cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const float v = element(w, i / w.cols, int(i % w.cols));
        if (!isfinite(v)) atomicExch(flag, 1);
    }
}

// One warp per row: shift = 15 - e where max|w| = m * 2^e, m in [0.5, 1).
__global__ void row_shift_kernel(DeviceMatrix w, signed char* out) {
    const long long r = blockIdx.x * (long long)(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= w.rows) return;
    float m = 0.f;
    for (int k = lane; k < w.cols; k += 32) m = fmaxf(m, fabsf(element(w, r, k)));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
        int e = 0;
        if (m > 0.f && isfinite(m)) frexpf(m, &e);
        out[r] = (signed char)(m > 0.f ? max(-100, min(100, 15 - e)) : 0);
    }
}

// Exact FP16 planes of a matrix: element value (the reference's dequantised
// F32) times 2^row_shift, split into hi + lo.
__global__ void planes_kernel(DeviceMatrix w, unsigned* hi, unsigned* lo) {
    const long long pairs = (long long)w.rows * w.cols / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < pairs; i += (long long)gridDim.x * blockDim.x) {
        const long long r = 2 * i / w.cols;
        const int k = int(2 * i % w.cols);
        const float f = __uint_as_float(unsigned(127 + w.row_shift[r]) << 23);
        split_exact(element(w, r, k) * f, element(w, r, k + 1) * f, hi[i], lo[i]);
    }
}

// Q4_K tensor-core form (DeviceMatrix::qplane ...) from the packed rows.
// Per row, the power of two that brings max |dmin * m| into [2^14, 2^15)
// (0 for a row without minima), so the split of dmin * m is exact.
__global__ void q4k_min_shift_kernel(DeviceMatrix w, signed char* out) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= w.rows) return;
    const unsigned char* meta = w.meta + (long long)r * w.meta_row;
    float mx = 0.f;
    for (int u = lane; u < w.cols / 32; u += 32) {
        const unsigned char* blk = meta + (u >> 3) * 16;
        unsigned sc, m;
        q4k_scale_min(blk + 4, u & 7, sc, m);
        mx = fmaxf(mx, fabsf(h2f((unsigned short)(blk[2] | (blk[3] << 8))) * float(m)));
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) {
        int e = 0;
        if (mx > 0.f) frexpf(mx, &e);
        out[r] = (signed char)(mx > 0.f ? 15 - e : 0);
    }
}

// qplane (pairs of sc*q), qscale (d per block), qmin_hi / qmin_lo (split of
// dmin * m * 2^shift per sub-block); one thread per pair of elements.
__global__ void q4k_planes_kernel(DeviceMatrix w, unsigned* qplane, float* qscale, unsigned short* min_hi,
                                  unsigned short* min_lo, const signed char* shift) {
    const long long pairs = (long long)w.rows * w.cols / 2;
    const int units = w.cols / 32;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < pairs; i += (long long)gridDim.x * blockDim.x) {
        const long long r = 2 * i / w.cols;
        const int k = int(2 * i % w.cols);
        const int u = k >> 5, j = k & 31;
        const unsigned char* blk = w.meta + r * (long long)w.meta_row + (k >> 8) * 16;
        unsigned sc, m;
        q4k_scale_min(blk + 4, u & 7, sc, m);
        const unsigned char* q = w.qs + r * (long long)w.qs_row + u * 16 + (j & 15);
        const unsigned q0 = j < 16 ? (q[0] & 15u) : (q[0] >> 4);
        const unsigned q1 = j < 16 ? (q[1] & 15u) : (q[1] >> 4);
        const __half2 p = __floats2half2_rn(float(sc * q0), float(sc * q1));  // integers < 1024: exact
        qplane[i] = *reinterpret_cast<const unsigned*>(&p);
        if (j == 0) {
            const float f = __uint_as_float(unsigned(127 + shift[r]) << 23);
            unsigned hi, lo;
            split_exact(h2f((unsigned short)(blk[2] | (blk[3] << 8))) * float(m) * f, 0.f, hi, lo);
            min_hi[r * units + u] = (unsigned short)(hi & 0xffffu);
            min_lo[r * units + u] = (unsigned short)(lo & 0xffffu);
        }
        if ((k & 255) == 0) qscale[r * (w.cols / 256) + (k >> 8)] = h2f((unsigned short)(blk[0] | (blk[1] << 8)));
    }
}

// Side arrays of the packed Q4_K tensor-core form (the codes stay in the
// packed rows): qsc, the 6-bit scale sc of every 32-element sub-block as a
// byte; qscale, d per 256-element block; qmin_hi / qmin_lo, the exact split of
// dmin * m * 2^shift per sub-block.  One thread per (row, sub-block).
__global__ void q4k_side_kernel(DeviceMatrix w, unsigned char* qsc, float* qscale, unsigned short* min_hi,
                                unsigned short* min_lo, const signed char* shift) {
    const int units = w.cols / 32;
    const long long n = (long long)w.rows * units;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / units;
        const int u = int(i % units);
        const unsigned char* blk = w.meta + r * (long long)w.meta_row + (u >> 3) * 16;
        unsigned sc, m;
        q4k_scale_min(blk + 4, u & 7, sc, m);
        qsc[i] = (unsigned char)sc;
        const float f = __uint_as_float(unsigned(127 + shift[r]) << 23);
        unsigned hi, lo;
        split_exact(h2f((unsigned short)(blk[2] | (blk[3] << 8))) * float(m) * f, 0.f, hi, lo);
        min_hi[i] = (unsigned short)(hi & 0xffffu);
        min_lo[i] = (unsigned short)(lo & 0xffffu);
        if ((u & 7) == 0) qscale[r * (w.cols / 256) + (u >> 3)] = h2f((unsigned short)(blk[0] | (blk[1] << 8)));
    }
}

__global__ void embed_kernel(DeviceMatrix w, const int* tokens, float* x, int ldx, int* ids, const int* blk,
                             const int* slot, int tpb) {
    const int t = blockIdx.x;
    const long long r = tokens[t];
    if (ids && threadIdx.x == 0) ids[(long long)blk[t] * tpb + slot[t]] = int(r);
    for (int k = threadIdx.x; k < w.cols; k += blockDim.x) x[(long long)t * ldx + k] = element(w, r, k);
}

// ----------------------------------------------------------------- GEMV
// x is staged in shared memory, padded by 4 floats every 128 so that the
// lanes of a quarter-warp read distinct banks, with the per-32 sums S that
// let the 4-bit kernels work on 1+q/16 instead of q (see dot_q4).
__host__ __device__ __forceinline__ int xpad(int k) { return k + ((k >> 7) << 2); }

// 8 nibbles of a word prepared as 0x80|q<<3 per byte, then one PRMT per
// nibble builds the float 1 + q/16 (exponent byte 0x3F, q in the top of the
// mantissa).  Exact for q in 0..15.
__device__ __forceinline__ float nib(unsigned prep, int k) {
    const unsigned sel = 5u | (5u << 4) | (unsigned(k) << 8) | (4u << 12);
    return __uint_as_float(__byte_perm(prep, 0x3Fu, sel));
}

// A = sum over a 32-element unit of (1 + q_e/16) * x_e.  Byte j of the unit:
// element j in the low nibble, element j+16 in the high nibble.
__device__ __forceinline__ float dot_q4_unit(uint4 w, const float* xs) {
    const unsigned ws[4] = {w.x, w.y, w.z, w.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const unsigned lo = ((ws[i] << 3) & 0x78787878u) | 0x80808080u;
        const unsigned hi = ((ws[i] >> 1) & 0x78787878u) | 0x80808080u;
        const float4 xl = *reinterpret_cast<const float4*>(xs + 4 * i);
        const float4 xh = *reinterpret_cast<const float4*>(xs + 16 + 4 * i);
        a0 = fmaf(nib(lo, 0), xl.x, a0);
        a1 = fmaf(nib(lo, 1), xl.y, a1);
        a0 = fmaf(nib(lo, 2), xl.z, a0);
        a1 = fmaf(nib(lo, 3), xl.w, a1);
        a0 = fmaf(nib(hi, 0), xh.x, a0);
        a1 = fmaf(nib(hi, 1), xh.y, a1);
        a0 = fmaf(nib(hi, 2), xh.z, a0);
        a1 = fmaf(nib(hi, 3), xh.w, a1);
    }
    return a0 + a1;
}

// sum over 16 int8 codes of q*x, q made exact with the 2^23 magic.
__device__ __forceinline__ float dot_q8_unit(uint4 w, const float* xs) {
    const unsigned ws[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + 4 * i);
        // byte k -> 0x4B0000bb = 2^23 + (q + 128); minus (2^23 + 128) = q exactly
        const float q0 = __uint_as_float(__byte_perm(ws[i], 0x4Bu, 0x4550u)) - 8388736.f;
        const float q1 = __uint_as_float(__byte_perm(ws[i], 0x4Bu, 0x4551u)) - 8388736.f;
        const float q2 = __uint_as_float(__byte_perm(ws[i], 0x4Bu, 0x4552u)) - 8388736.f;
        const float q3 = __uint_as_float(__byte_perm(ws[i], 0x4Bu, 0x4553u)) - 8388736.f;
        a0 = fmaf(q0, xv.x, a0);
        a1 = fmaf(q1, xv.y, a1);
        a0 = fmaf(q2, xv.z, a0);
        a1 = fmaf(q3, xv.w, a1);
    }
    return a0 + a1;
}

template <int TYPE>
struct Unit {
    // elements per 16-byte unit of qs
    static constexpr int kElems = TYPE == kQ8_0 ? 16 : (TYPE == kF16 ? 8 : (TYPE == kF32 ? 4 : 32));
};

template <int TYPE>
__device__ __forceinline__ float unit_dot(uint4 w, const float* xs, float s, int u, const unsigned char* meta) {
    if constexpr (TYPE == kQ8_0) {
        const float d = h2f(reinterpret_cast<const unsigned short*>(meta)[u >> 1]);
        return d * dot_q8_unit(w, xs);
    } else if constexpr (TYPE == kQ4_0) {
        const float d = h2f(reinterpret_cast<const unsigned short*>(meta)[u]);
        // sum d*(q-8)*x = d*(16*A - 24*S)
        return d * fmaf(16.f, dot_q4_unit(w, xs), -24.f * s);
    } else if constexpr (TYPE == kQ4_K) {
        const uint4 m = __ldg(reinterpret_cast<const uint4*>(meta) + (u >> 3));
        const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xffff)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
        float sc, mn;
        q4k_scale_min_w(m.y, m.z, m.w, u & 7, sc, mn);
        // sum (d*sc*q - dmin*m)*x = 16*d*sc*A - (16*d*sc + dmin*m)*S
        const float ds = 16.f * d * sc;
        return fmaf(ds, dot_q4_unit(w, xs), -fmaf(dmin, mn, ds) * s);
    } else if constexpr (TYPE == kF16) {
        const __half2* h = reinterpret_cast<const __half2*>(&w);
        const float4 x0 = *reinterpret_cast<const float4*>(xs);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + 4);
        const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]),
                     e = __half22float2(h[3]);
        float r = a.x * x0.x;
        r = fmaf(a.y, x0.y, r);
        r = fmaf(b.x, x0.z, r);
        r = fmaf(b.y, x0.w, r);
        r = fmaf(c.x, x1.x, r);
        r = fmaf(c.y, x1.y, r);
        r = fmaf(e.x, x1.z, r);
        return fmaf(e.y, x1.w, r);
    } else {
        const float4 x0 = *reinterpret_cast<const float4*>(xs);
        float r = __uint_as_float(w.x) * x0.x;
        r = fmaf(__uint_as_float(w.y), x0.y, r);
        r = fmaf(__uint_as_float(w.z), x0.z, r);
        return fmaf(__uint_as_float(w.w), x0.w, r);
    }
}

// The unit u of R rows against one token's x: each float4 of x is read from
// shared memory once and used for all R rows (the x traffic per weight byte
// falls by R).  Same arithmetic per row as unit_dot.
template <int TYPE, int R>
__device__ __forceinline__ void rows_unit_dot(const uint4 (&wv)[R], const float* xs, float s, int u,
                                              const unsigned char* const (&meta)[R], float (&acc)[R]) {
    if constexpr (TYPE == kQ4_0 || TYPE == kQ4_K) {
        float a0[R], a1[R];
#pragma unroll
        for (int r = 0; r < R; ++r) a0[r] = a1[r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 xl = *reinterpret_cast<const float4*>(xs + 4 * i);
            const float4 xh = *reinterpret_cast<const float4*>(xs + 16 + 4 * i);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned w = i == 0 ? wv[r].x : i == 1 ? wv[r].y : i == 2 ? wv[r].z : wv[r].w;
                const unsigned lo = ((w << 3) & 0x78787878u) | 0x80808080u;
                const unsigned hi = ((w >> 1) & 0x78787878u) | 0x80808080u;
                a0[r] = fmaf(nib(lo, 0), xl.x, a0[r]);
                a1[r] = fmaf(nib(lo, 1), xl.y, a1[r]);
                a0[r] = fmaf(nib(lo, 2), xl.z, a0[r]);
                a1[r] = fmaf(nib(lo, 3), xl.w, a1[r]);
                a0[r] = fmaf(nib(hi, 0), xh.x, a0[r]);
                a1[r] = fmaf(nib(hi, 1), xh.y, a1[r]);
                a0[r] = fmaf(nib(hi, 2), xh.z, a0[r]);
                a1[r] = fmaf(nib(hi, 3), xh.w, a1[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float A = a0[r] + a1[r];
            if constexpr (TYPE == kQ4_0) {
                const float d = h2f(reinterpret_cast<const unsigned short*>(meta[r])[u]);
                acc[r] += d * fmaf(16.f, A, -24.f * s);
            } else {
                const uint4 m = __ldg(reinterpret_cast<const uint4*>(meta[r]) + (u >> 3));
                const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xffff)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
                float sc, mn;
                q4k_scale_min_w(m.y, m.z, m.w, u & 7, sc, mn);
                const float ds = 16.f * d * sc;
                acc[r] += fmaf(ds, A, -fmaf(dmin, mn, ds) * s);
            }
        }
    } else if constexpr (TYPE == kQ8_0) {
        float a0[R], a1[R];
#pragma unroll
        for (int r = 0; r < R; ++r) a0[r] = a1[r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 xv = *reinterpret_cast<const float4*>(xs + 4 * i);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned w = (i == 0 ? wv[r].x : i == 1 ? wv[r].y : i == 2 ? wv[r].z : wv[r].w) ^ 0x80808080u;
                a0[r] = fmaf(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u)) - 8388736.f, xv.x, a0[r]);
                a1[r] = fmaf(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4551u)) - 8388736.f, xv.y, a1[r]);
                a0[r] = fmaf(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4552u)) - 8388736.f, xv.z, a0[r]);
                a1[r] = fmaf(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4553u)) - 8388736.f, xv.w, a1[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
            acc[r] += h2f(reinterpret_cast<const unsigned short*>(meta[r])[u >> 1]) * (a0[r] + a1[r]);
    } else {
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += unit_dot<TYPE>(wv[r], xs, s, u, meta[r]);
    }
}

// The reference SwiGLU (model.hpp:120-124): gate * (sigmoid(gate) * up).
__device__ __forceinline__ float swiglu(float g, float up) {
    const float small = expf(-fabsf(g));
    const float sig = g >= 0.f ? 1.f / (1.f + small) : small / (1.f + small);
    return __fmul_rn(g, __fmul_rn(sig, up));
}

// R rows per warp, NT tokens per pass; each warp streams its rows once per
// pass over the K chunk held in shared memory.
template <int TYPE, int R, int NT>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(GemmArgs a, int kc) {
    extern __shared__ float smem[];
    constexpr int E = Unit<TYPE>::kElems;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    const int K = a.w.cols;
    const int kcp = xpad(kc);  // padded chunk stride
    float* xs = smem;                 // [NT][kcp]
    float* s32 = smem + NT * kcp;     // [NT][kc/32]
    for (int t0 = 0; t0 < a.tokens; t0 += NT) {
        const int nt = min(NT, a.tokens - t0);
        float acc[R][NT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        for (int k0 = 0; k0 < K; k0 += kc) {
            const int klen = min(kc, K - k0);
            __syncthreads();
            for (int i = threadIdx.x; i < NT * (klen / 4); i += blockDim.x) {
                const int t = i / (klen / 4), k = (i % (klen / 4)) * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < nt) v = __ldg(reinterpret_cast<const float4*>(a.x + (long long)(t0 + t) * a.ldx + k0 + k));
                *reinterpret_cast<float4*>(xs + t * kcp + xpad(k)) = v;
            }
            __syncthreads();
            if (TYPE == kQ4_0 || TYPE == kQ4_K) {
                for (int i = threadIdx.x; i < NT * (klen / 32); i += blockDim.x) {
                    const int t = i / (klen / 32), g = i % (klen / 32);
                    const float* p = xs + t * kcp + xpad(g * 32);
                    float s = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) s += p[j];
                    s32[t * (kc / 32) + g] = s;
                }
                __syncthreads();
            }
            if (row0 < a.w.rows) {
                const int units = klen / E, ubase = k0 / E;
#pragma unroll 2
                for (int u = lane; u < units; u += 32) {
                    uint4 wv[R];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int row = min(row0 + r, a.w.rows - 1);
                        wv[r] = ld_stream(a.w.qs + (long long)row * a.w.qs_row + (long long)(ubase + u) * 16);
                    }
                    const unsigned char* metas[R];
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        metas[r] = a.w.meta + (long long)min(row0 + r, a.w.rows - 1) * a.w.meta_row;
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        if (t < nt) {
                            const float* xp = xs + t * kcp + xpad(u * E);
                            const float sv = (TYPE == kQ4_0 || TYPE == kQ4_K) ? s32[t * (kc / 32) + u] : 0.f;
                            float col[R];
#pragma unroll
                            for (int r = 0; r < R; ++r) col[r] = acc[r][t];
                            rows_unit_dot<TYPE, R>(wv, xp, sv, ubase + u, metas, col);
#pragma unroll
                            for (int r = 0; r < R; ++r) acc[r][t] = col[r];
                        }
                    }
                }
            }
        }
        if (row0 < a.w.rows) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float v = acc[r][t];
#pragma unroll
                    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    acc[r][t] = v;
                }
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= nt) continue;
                    float* y = a.y + (long long)(t0 + t) * a.ldy;
                    if (a.epilogue == kSwiGLU) {
#pragma unroll
                        for (int r = 0; r + 1 < R; r += 2)
                            if (row0 + r + 1 < a.w.rows) y[(row0 + r) / 2] = swiglu(acc[r][t], acc[r + 1][t]);
                    } else {
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            if (row0 + r >= a.w.rows) continue;
                            if (a.epilogue == kAdd) y[row0 + r] += acc[r][t];
                            else y[row0 + r] = acc[r][t];
                        }
                    }
                }
            }
        }
    }
}

// One token (decode): no shared-memory staging, so no barrier delays the
// first weight loads.  Warp = kRows1 rows; lane l takes units l, l+32, ... of
// them, prefetching the next unit's loads while it computes the current one.
// The unit's x is read float4 by float4 through L1 (each load serves all the
// warp's rows) and, for the 4-bit types, summed on the way.  Few live
// registers (row addresses from one base, x never held whole), so many warps
// stay resident to hide the load latency.
constexpr int kRows1 = 4;

// Packed F32x2 arithmetic (Blackwell fma.rn.f32x2 / add.rn.f32x2): two
// weights per instruction, each half rounded exactly as the scalar op.
__device__ __forceinline__ unsigned long long f2pk(float x, float y) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ float f2sum(unsigned long long r) {
    float x, y;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(r));
    return x + y;
}
__device__ __forceinline__ unsigned long long f2fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// x of unit u staged transposed in shared memory: float4 #i of unit u at
// xt[i * units + u], so the lanes of a warp (consecutive units) read
// consecutive 16-byte words.  S[u] = sum of the unit's x (4-bit types).
template <int TYPE>
__device__ __forceinline__ void rows_unit_dot_t(const uint4 (&wv)[kRows1], const float4* xt, int units, float S,
                                                int u, const unsigned char* meta0, std::size_t meta_row,
                                                float (&acc)[kRows1]) {
    constexpr int R = kRows1;
    if constexpr (TYPE == kQ4_0 || TYPE == kQ4_K) {
        unsigned long long a2[R];
#pragma unroll
        for (int r = 0; r < R; ++r) a2[r] = 0ull;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 xl = xt[i * units + u];
            const float4 xh = xt[(4 + i) * units + u];
            const unsigned long long l01 = f2pk(xl.x, xl.y), l23 = f2pk(xl.z, xl.w);
            const unsigned long long h01 = f2pk(xh.x, xh.y), h23 = f2pk(xh.z, xh.w);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned w = i == 0 ? wv[r].x : i == 1 ? wv[r].y : i == 2 ? wv[r].z : wv[r].w;
                const unsigned lo = ((w << 3) & 0x78787878u) | 0x80808080u;
                const unsigned hi = ((w >> 1) & 0x78787878u) | 0x80808080u;
                a2[r] = f2fma(f2pk(nib(lo, 0), nib(lo, 1)), l01, a2[r]);
                a2[r] = f2fma(f2pk(nib(lo, 2), nib(lo, 3)), l23, a2[r]);
                a2[r] = f2fma(f2pk(nib(hi, 0), nib(hi, 1)), h01, a2[r]);
                a2[r] = f2fma(f2pk(nib(hi, 2), nib(hi, 3)), h23, a2[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const unsigned char* meta = meta0 + r * meta_row;
            const float A = f2sum(a2[r]);
            if constexpr (TYPE == kQ4_0) {
                const float d = h2f(reinterpret_cast<const unsigned short*>(meta)[u]);
                acc[r] += d * fmaf(16.f, A, -24.f * S);
            } else {
                const uint4 m = __ldg(reinterpret_cast<const uint4*>(meta) + (u >> 3));
                const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xffff)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
                float sc, mn;
                q4k_scale_min_w(m.y, m.z, m.w, u & 7, sc, mn);
                const float ds = 16.f * d * sc;
                acc[r] += fmaf(ds, A, -fmaf(dmin, mn, ds) * S);
            }
        }
    } else if constexpr (TYPE == kQ8_0) {
        unsigned long long a2[R];
        const unsigned long long bias = f2pk(-8388736.f, -8388736.f);  // -(2^23 + 128)
#pragma unroll
        for (int r = 0; r < R; ++r) a2[r] = 0ull;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 xv = xt[i * units + u];
            const unsigned long long x01 = f2pk(xv.x, xv.y), x23 = f2pk(xv.z, xv.w);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const unsigned w = (i == 0 ? wv[r].x : i == 1 ? wv[r].y : i == 2 ? wv[r].z : wv[r].w) ^ 0x80808080u;
                const unsigned long long q01 = f2add(f2pk(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u)),
                                                          __uint_as_float(__byte_perm(w, 0x4Bu, 0x4551u))), bias);
                const unsigned long long q23 = f2add(f2pk(__uint_as_float(__byte_perm(w, 0x4Bu, 0x4552u)),
                                                          __uint_as_float(__byte_perm(w, 0x4Bu, 0x4553u))), bias);
                a2[r] = f2fma(q01, x01, a2[r]);
                a2[r] = f2fma(q23, x23, a2[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
            acc[r] += h2f(reinterpret_cast<const unsigned short*>(meta0 + r * meta_row)[u >> 1]) * f2sum(a2[r]);
    } else {
        alignas(16) float xv[Unit<TYPE>::kElems];
#pragma unroll
        for (int j = 0; j < Unit<TYPE>::kElems / 4; ++j) {
            const float4 v = xt[j * units + u];
            xv[4 * j] = v.x;
            xv[4 * j + 1] = v.y;
            xv[4 * j + 2] = v.z;
            xv[4 * j + 3] = v.w;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += unit_dot<TYPE>(wv[r], xv, 0.f, u, meta0 + r * meta_row);
    }
}

// Integer path of the quantised formats (streamed GEMV).  Each unit of the
// token's x is held as 22-bit fixed point against the unit's own max:
// x_int = rint(x * 2^sh) with max |x| * 2^sh in [2^21, 2^22), so each x is
// rounded by at most 2^-22 of its unit's max |x| (the reference's own
// quantised dot products, quant.hpp:87-161, round x to 8 bits per block).  Its two's-complement bytes are the digits, x_int = b0 + 256 b1 +
// 65536 b2 with b0, b1 unsigned and b2 = x_int >> 16 signed (|b2| <= 64), so
// no carries need fixing.  Digit words hold one byte position of four
// consecutive elements: d[k][w] = digit k of elements 16w..16w+15.  The codes
// of a weight word (four int8, or eight nibbles as two masked words) meet the
// digit words in dp4a, three per four codes; the partial sums stay below
// 2^20, so (S0 + 256 S1 + 65536 S2) * 2^-sh is sum(q * x) to float rounding,
// and the block scale is applied once per unit.  A lane keeps the digits of
// the units it works on in registers for the whole launch.
__device__ __forceinline__ float small_int_to_float(int v) {  // exact for |v| < 2^22
    return __int_as_float(v + 0x4B400000) - 12582912.f;
}
__device__ __forceinline__ int dp4a_uu(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int TYPE>
struct XUnit {
    static constexpr int kW4 = Unit<TYPE>::kElems / 16;
    uint4 d[3][kW4];  // digit words (see above)
    float S;          // sum of the unit's x
    float inv;        // 2^-sh
};

// One unit of x in the form above.  A unit whose max |x| is inf or NaN gets
// inv = NaN, so its products come out NaN.
template <int TYPE>
__device__ __forceinline__ void load_xunit(const float* x, int u, XUnit<TYPE>& xu) {
    constexpr int E = Unit<TYPE>::kElems, F4 = E / 4, W4 = E / 16;
    float4 v[F4];
    float sum = 0.f, mx = 0.f;
#pragma unroll
    for (int j = 0; j < F4; ++j) {
        v[j] = __ldg(reinterpret_cast<const float4*>(x + (long long)u * E) + j);
        sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    }
    // mx = m * 2^e with m in [0.5, 1); zero and subnormal units take the clamp
    const int e = int((__float_as_uint(mx) >> 23) & 255u) - 126;
    const int sh = min(126, 22 - e);  // e <= 128: 2^sh and 2^-sh stay normal
    const bool fin = mx <= 3.4028235e38f;  // false for inf and NaN
    const float up = fin ? __uint_as_float(unsigned(127 + sh) << 23) : 0.f;
    xu.S = sum;
    xu.inv = fin ? __uint_as_float(unsigned(127 - sh) << 23) : mx - mx;
#pragma unroll
    for (int w = 0; w < W4; ++w) {
        unsigned b[3][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 f = v[w * 4 + q];
            // round to nearest integer through the 1.5 * 2^23 magic (|x * 2^sh| <= 2^22)
            const unsigned i0 = __float_as_uint(fmaf(f.x, up, 12582912.f)) - 0x4B400000u;
            const unsigned i1 = __float_as_uint(fmaf(f.y, up, 12582912.f)) - 0x4B400000u;
            const unsigned i2 = __float_as_uint(fmaf(f.z, up, 12582912.f)) - 0x4B400000u;
            const unsigned i3 = __float_as_uint(fmaf(f.w, up, 12582912.f)) - 0x4B400000u;
            const unsigned lo01 = __byte_perm(i0, i1, 0x5140);  // i0.b0 i1.b0 i0.b1 i1.b1
            const unsigned lo23 = __byte_perm(i2, i3, 0x5140);
            const unsigned hi01 = __byte_perm(i0, i1, 0x0062);  // i0.b2 i1.b2 . .
            const unsigned hi23 = __byte_perm(i2, i3, 0x0062);
            b[0][q] = __byte_perm(lo01, lo23, 0x5410);
            b[1][q] = __byte_perm(lo01, lo23, 0x7632);
            b[2][q] = __byte_perm(hi01, hi23, 0x5410);
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) xu.d[k][w] = make_uint4(b[k][0], b[k][1], b[k][2], b[k][3]);
    }
}

// Q4_K scale and min of sub-block g from the three scale words, with the
// shifts and masks fixed per lane (a lane always sees the same g).
struct Q4kSel {
    unsigned sh, sh2, ma, mb;
    bool hi;
    __device__ __forceinline__ explicit Q4kSel(int g) {
        hi = g >= 4;
        sh = 8u * unsigned(g & 3);
        sh2 = sh + 2u;
        ma = hi ? 15u : 63u;
        mb = hi ? 0x30u : 0u;
    }
    // sub-blocks 0-3: (y & 63, z & 63); 4-7: (w & 15 | (y >> 6) << 4, w >> 4 | (z >> 6) << 4)
    __device__ __forceinline__ void decode(unsigned y, unsigned z, unsigned w, float& sc, float& mn) const {
        const unsigned a = ((hi ? w : y) >> sh) & ma;
        const unsigned b = ((hi ? (w >> 4) : z) >> sh) & ma;
        sc = __uint_as_float(a | ((y >> sh2) & mb) | 0x4B000000u) - 8388608.f;
        mn = __uint_as_float(b | ((z >> sh2) & mb) | 0x4B000000u) - 8388608.f;
    }
};

// acc[r] += row r's unit (codes wv[r], block headers at meta0 + r * meta_row,
// unit mu of them) . x unit xu.
template <int TYPE>
__device__ __forceinline__ void rows_unit_dot_x(const uint4 (&wv)[kRows1], const XUnit<TYPE>& xu,
                                                const unsigned char* meta0, int meta_row, int mu, const Q4kSel& sel,
                                                float (&acc)[kRows1]) {
    auto word = [](const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; };
#pragma unroll
    for (int r = 0; r < kRows1; ++r) {
        int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const unsigned w = word(wv[r], i);
            if constexpr (TYPE == kQ8_0) {
                // elements 4i..4i+3: digit word i of the unit's 16
                s0 = dp4a_su(w, word(xu.d[0][0], i), s0);
                s1 = dp4a_su(w, word(xu.d[1][0], i), s1);
                s2 = dp4a_ss(w, word(xu.d[2][0], i), s2);
            } else {
                // low nibbles: elements 4i..4i+3 (digit word i of 0..15);
                // high nibbles: elements 16+4i.. (digit word i of 16..31)
                const unsigned lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
                s0 = dp4a_uu(lo, word(xu.d[0][0], i), dp4a_uu(hi, word(xu.d[0][1], i), s0));
                s1 = dp4a_uu(lo, word(xu.d[1][0], i), dp4a_uu(hi, word(xu.d[1][1], i), s1));
                s2 = dp4a_us(lo, word(xu.d[2][0], i), dp4a_us(hi, word(xu.d[2][1], i), s2));
            }
        }
        // sum(q * x) = (S0 + 256 (S1 + 256 S2)) * 2^-sh (S1 + 256 S2 < 2^26: one
        // rounding in its conversion, S0 converts exactly)
        const float A = fmaf(256.f, float(s1 + 256 * s2), small_int_to_float(s0)) * xu.inv;
        const unsigned char* meta = meta0 + r * meta_row;
        if constexpr (TYPE == kQ8_0) {
            acc[r] = fmaf(h2f(reinterpret_cast<const unsigned short*>(meta)[mu >> 1]), A, acc[r]);
        } else if constexpr (TYPE == kQ4_0) {
            const float d = h2f(reinterpret_cast<const unsigned short*>(meta)[mu]);
            acc[r] = fmaf(d, fmaf(-8.f, xu.S, A), acc[r]);
        } else {
            const uint4 m = reinterpret_cast<const uint4*>(meta)[mu >> 3];
            const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xffff)));
            const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
            float sc, mn;
            sel.decode(m.y, m.z, m.w, sc, mn);
            acc[r] = fmaf(d * sc, A, fmaf(-dmin * mn, xu.S, acc[r]));
        }
    }
}

template <int TYPE>
__global__ void __launch_bounds__(kWarps * 32) gemv1_kernel(GemmArgs a) {
    constexpr int R = kRows1, E = Unit<TYPE>::kElems, F4 = E / 4;
    extern __shared__ float4 gemv_xt[];  // [F4][units] transposed x, then S[units]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int units = a.w.cols / E;
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    const bool active = row0 < a.w.rows;
    // The last group starts R rows before the end instead of reading past it
    // (it recomputes rows of the previous group and stores only its own).
    // The launcher sends matrices of fewer than R rows elsewhere.
    const int base_row = min(row0, a.w.rows - R);
    const int shift_rows = row0 - base_row;
    const unsigned char* q0 = a.w.qs + (long long)base_row * a.w.qs_row;
    const unsigned char* m0 = a.w.meta + (long long)base_row * a.w.meta_row;
    constexpr int kAhead = 2;  // units of weight loads in flight per lane
    uint4 ring[kAhead][R];
    // weight loads first: they are in flight while x is staged
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
        const int u = lane + 32 * j;
#pragma unroll
        for (int r = 0; r < R; ++r)
            ring[j][r] = active && u < units ? ld_stream(q0 + r * a.w.qs_row + (long long)u * 16) : make_uint4(0, 0, 0, 0);
    }
    // Programmatic dependent launch: the weights above do not depend on the
    // previous kernel, x does.  Let the next kernel start its own prefetch
    // (it launches once every CTA of this grid has reached this point), then
    // wait for the previous kernel's results before reading x.  Both are
    // no-ops for an ordinary launch.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float* S = reinterpret_cast<float*>(gemv_xt + F4 * units);
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < F4; ++j) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(a.x + (long long)u * E) + j);
            gemv_xt[j * units + u] = v;
            sum += (v.x + v.y) + (v.z + v.w);
        }
        S[u] = sum;
    }
    __syncthreads();
    if (!active) return;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int u0 = lane; u0 < units; u0 += 32 * kAhead) {
#pragma unroll
        for (int j = 0; j < kAhead; ++j) {
            const int u = u0 + 32 * j;
            if (u >= units) break;
            // refill the slot before computing on its old contents, so the
            // next load is in flight during this unit's arithmetic
            uint4 cur[R];
#pragma unroll
            for (int r = 0; r < R; ++r) cur[r] = ring[j][r];
            const int un = u + 32 * kAhead;
            if (un < units) {
#pragma unroll
                for (int r = 0; r < R; ++r) ring[j][r] = ld_stream(q0 + r * a.w.qs_row + (long long)un * 16);
            }
            rows_unit_dot_t<TYPE>(cur, gemv_xt, units, S[u], u, m0, a.w.meta_row, acc);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    if (lane == 0) {
        // results for rows base_row + r; this group owns rows row0.. (r >= shift_rows)
        if (a.epilogue == kSwiGLU) {
#pragma unroll
            for (int r = 0; r + 1 < R; r += 2)
                if (r >= shift_rows && base_row + r + 1 < a.w.rows)
                    a.y[(base_row + r) / 2] = swiglu(acc[r], acc[r + 1]);
        } else {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (r < shift_rows || base_row + r >= a.w.rows) continue;
                if (a.epilogue == kAdd) a.y[base_row + r] += acc[r];
                else a.y[base_row + r] = acc[r];
            }
        }
    }
}

// ------------------------------------------------------------ streamed GEMV
// Single-token projection of a quantised matrix with the weights streamed
// through shared memory.  A copy warp moves each stage -- the codes and block
// headers of RG rows over KCU units of K -- with cp.async.bulk (one copy per
// row and array) onto the stage's mbarrier, stream_stages() stages ahead,
// starting before the wait on the previous kernel since the weights do not
// depend on it.  Eight consumer warps compute from shared memory: a lane owns
// one unit position of the stage for a set of four rows, so it sees the same
// CH units of x (one per K chunk) in every row group and keeps their digits
// in registers for the whole launch.  RG = 1024 / KCU rows per stage (16 KB
// of codes); the grid is persistent and takes row groups in turn.  Every wait
// is bounded; on a timeout the kernel records an error, stops issuing copies,
// keeps its barriers in step, waits (bounded) for the copies it issued and
// exits.
constexpr int kStreamWarps = 8;                          // consumer warps
constexpr int kStreamThreads = (kStreamWarps + 1) * 32;  // + the copy warp
constexpr int kStreamSlots = kStreamWarps * 32;          // (unit, 4-row set) slots per stage
// Stages per CTA: six of 18 KB for the 4-bit formats keep two CTAs per SM
// (2 x 108 KB of the SM's 228 KB), so an 11008 x 4096 Q4_K or Q4_0 matrix
// (172 KB per SM) is requested whole at launch; Q8_0 (twice the bytes per
// row) measured faster with four.
template <int TYPE>
constexpr int stream_stages() { return TYPE == kQ8_0 ? 4 : 6; }
constexpr int kStreamQs = kStreamSlots * 4 * 16;         // 16 KB of codes per stage
constexpr int kStreamMeta = kStreamSlots * 4 * 2;        // block headers: <= 2 bytes per unit
constexpr unsigned kStreamSpin = 1u << 24;

__device__ int g_gemv_stream_err;  // error word when the caller passed none

struct StreamShape {
    int kcu;     // units per row per stage: a power of two in [32, 256]
    int rg;      // rows per group (1024 / kcu)
    int chunks;  // stages per row group
    int groups;  // row groups
};

__device__ __forceinline__ unsigned sh_addr(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void sb_init(std::uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sh_addr(bar)), "r"(count));
}
__device__ __forceinline__ void sb_arrive(std::uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sh_addr(bar)) : "memory");
}
__device__ __forceinline__ void sb_expect(std::uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sh_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool sb_try(std::uint64_t* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(sh_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void sb_copy(void* dst, const void* src, unsigned bytes, std::uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sh_addr(dst)),
                 "l"(src), "r"(bytes), "r"(sh_addr(bar))
                 : "memory");
}
// Bounded wait: false on timeout (the error code is recorded and the abort
// flag set) or, when abort_flag is given, once another warp has given up.
__device__ __forceinline__ bool sb_wait(std::uint64_t* bar, unsigned parity, volatile int* abort_flag, int* err,
                                        int code) {
    for (unsigned i = 0; i < kStreamSpin; ++i) {
        if (sb_try(bar, parity)) return true;
        if (abort_flag && *abort_flag) return false;
        if (i > 16) __nanosleep(64);
    }
    if (abort_flag) *abort_flag = 1;
    atomicExch(err, code);
    return false;
}

template <int TYPE, int CH>
__global__ void __launch_bounds__(kStreamThreads, 2) gemv_stream_kernel(GemmArgs a, StreamShape sp) {
    constexpr int E = Unit<TYPE>::kElems;
    constexpr int MPU = TYPE == kQ8_0 ? 1 : 2;  // block-header bytes per unit
    constexpr int kSt = stream_stages<TYPE>();
    // [stages][16 KB] codes, then [stages][2 KB] headers
    extern __shared__ __align__(16) unsigned char stream_smem[];
    unsigned char* st_qs = stream_smem;
    unsigned char* st_meta = stream_smem + kSt * kStreamQs;
    __shared__ std::uint64_t full[kSt], empty[kSt];
    __shared__ float red[kSt][kStreamWarps][4];
    __shared__ int abort_word;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = a.w.cols / E;
    int* err = a.err ? a.err : &g_gemv_stream_err;
    volatile int* abort_flag = &abort_word;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSt; ++i) {
            sb_init(&full[i], 1);
            sb_init(&empty[i], kStreamWarps);
        }
        abort_word = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == kStreamWarps) {  // copy warp
        int it = 0;
        for (int g = blockIdx.x; g < sp.groups; g += gridDim.x) {
            const int row0 = g * sp.rg;
            const int nr = min(sp.rg, a.w.rows - row0);
            bool ok = true;
            for (int c = 0; c < sp.chunks; ++c) {
                const int st = it % kSt;
                const unsigned ph = (unsigned(it) / kSt) & 1u;
                int go = lane == 0 ? int(sb_wait(&empty[st], ph ^ 1u, abort_flag, err, 21)) : 0;
                go = __shfl_sync(0xffffffffu, go, 0);
                if (!go) {
                    ok = false;
                    break;
                }
                const int cu = min(sp.kcu, units - c * sp.kcu);
                if (lane == 0) sb_expect(&full[st], unsigned(nr * cu * (16 + MPU)));
                __syncwarp();
                if (lane < nr) {
                    const long long row = row0 + lane;
                    sb_copy(st_qs + st * kStreamQs + lane * sp.kcu * 16,
                            a.w.qs + row * (long long)a.w.qs_row + (long long)c * sp.kcu * 16, unsigned(cu * 16),
                            &full[st]);
                    sb_copy(st_meta + st * kStreamMeta + lane * sp.kcu * MPU,
                            a.w.meta + row * (long long)a.w.meta_row + (long long)c * sp.kcu * MPU, unsigned(cu * MPU),
                            &full[st]);
                }
                ++it;
            }
            if (!ok) break;
        }
        // the copies issued land before the CTA exits (bounded, even after an abort)
        if (lane == 0)
            for (int j = max(0, it - kSt); j < it; ++j)
                sb_wait(&full[j % kSt], (unsigned(j) / kSt) & 1u, nullptr, err, 22);
        return;
    }

    // consumer warps: x depends on the previous kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ul = threadIdx.x & (sp.kcu - 1);  // unit within the stage
    const int rs = threadIdx.x / sp.kcu;        // 4-row set within the group (one per warp or warp range)
    const int wpr = sp.kcu / 32;                // warps per 4-row set
    XUnit<TYPE> xu[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c)
        if (c * sp.kcu + ul < units) load_xunit<TYPE>(a.x, c * sp.kcu + ul, xu[c]);
    const Q4kSel sel(ul & 7);  // stage offsets are multiples of 8 units
    // this warp's sums for the rows of stage st (one unit of K, four rows)
    auto stage_dot = [&](int st, int c, float (&acc)[kRows1]) {
        if (c * sp.kcu + ul < units) {
            const unsigned char* q = st_qs + st * kStreamQs + (rs * 4 * sp.kcu + ul) * 16;
            uint4 wv[kRows1];
#pragma unroll
            for (int r = 0; r < kRows1; ++r) wv[r] = *reinterpret_cast<const uint4*>(q + r * sp.kcu * 16);
            rows_unit_dot_x<TYPE>(wv, xu[c], st_meta + st * kStreamMeta + rs * 4 * sp.kcu * MPU, sp.kcu * MPU, ul,
                                  sel, acc);
        }
    };
    // group g's rows from the warps' partial sums in red[slot] (one warp, lane = row)
    auto group_out = [&](int g, int slot) {
        float v = 0.f;
        if (lane < sp.rg)
            for (int w = 0; w < wpr; ++w) v += red[slot][(lane >> 2) * wpr + w][lane & 3];
        const float partner = __shfl_down_sync(0xffffffffu, v, 1);
        const int row = g * sp.rg + lane;
        if (lane < sp.rg && row < a.w.rows) {
            if (a.epilogue == kSwiGLU) {
                if (!(lane & 1)) a.y[row / 2] = swiglu(v, partner);
            } else if (a.epilogue == kAdd) {
                a.y[row] += v;
            } else {
                a.y[row] = v;
            }
        }
    };
    const int mine = (sp.groups - 1 - int(blockIdx.x)) / int(gridDim.x) + 1;  // groups of this CTA
    if (CH == 1 && mine <= kSt) {
        // Every group of this CTA has a stage of its own, filled once (phase
        // 0): take the stages in the order they land, keep each warp's sums
        // per stage and reduce all the groups after one barrier.  A stage
        // counts as landed when every lane has observed its barrier.
        unsigned done = 0;
        int left = mine;
        for (unsigned spin = 0; left > 0;) {
            bool moved = false;
            for (int j = 0; j < mine; ++j) {
                if ((done >> j) & 1u) continue;
                if (!__all_sync(0xffffffffu, sb_try(&full[j], 0u))) continue;
                float acc[kRows1] = {0.f, 0.f, 0.f, 0.f};
                stage_dot(j, 0, acc);
#pragma unroll
                for (int r = 0; r < kRows1; ++r)
#pragma unroll
                    for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
                if (lane == 0) {
#pragma unroll
                    for (int r = 0; r < kRows1; ++r) red[j][warp][r] = acc[r];
                }
                done |= 1u << j;
                --left;
                moved = true;
            }
            if (moved) continue;
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            if (++spin >= kStreamSpin) {
                *abort_flag = 1;
                if (lane == 0) atomicExch(err, 23);
                break;
            }
            __nanosleep(64);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kStreamSlots) : "memory");
        if (warp < mine) group_out(int(blockIdx.x) + warp * int(gridDim.x), warp);
        return;
    }
    int it = 0, gi = 0;
    for (int g = blockIdx.x; g < sp.groups; g += gridDim.x, ++gi) {
        float acc[kRows1] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < CH; ++c, ++it) {
            const int st = it % kSt;
            const unsigned ph = (unsigned(it) / kSt) & 1u;
            // after an abort the warps keep the same steps (no early exit) so
            // every barrier below is still reached by all of them
            if (!*abort_flag) sb_wait(&full[st], ph, abort_flag, err, 23);
            stage_dot(st, c, acc);
            __syncwarp();
            if (lane == 0) sb_arrive(&empty[st]);
        }
#pragma unroll
        for (int r = 0; r < kRows1; ++r)
#pragma unroll
            for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < kRows1; ++r) red[gi & 1][warp][r] = acc[r];
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kStreamSlots) : "memory");
        // red is double-buffered by group, so the next group's partial sums
        // do not overwrite these
        if (warp == 0) group_out(g, gi & 1);
    }
}

template <int TYPE, int R, int NT>
void run_gemv(const GemmArgs& a, cudaStream_t s) {
    constexpr int E = Unit<TYPE>::kElems;
    // K chunk: largest multiple of 256 whose staged activations fit 48 KB.
    const int budget = 48 * 1024;
    int kc = (budget / (NT * 4)) * 128 / 136 / 256 * 256;  // padding of 4 per 128
    kc = kc - kc % 256;
    if (kc >= a.w.cols) kc = a.w.cols;
    (void)E;
    const std::size_t smem = std::size_t(NT) * (xpad(kc) + kc / 32 + 4) * sizeof(float);
    const int rows_per_cta = kWarps * R;
    const int grid = (a.w.rows + rows_per_cta - 1) / rows_per_cta;
    gemv_kernel<TYPE, R, NT><<<grid, kWarps * 32, smem, s>>>(a, kc);
    TVARA_LAUNCHED();
}

int gemv_sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < 64 && cached[dev]) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev < 64) cached[dev] = n;
    return n;
}

template <int TYPE, int CH>
bool launch_gemv_stream_ch(const GemmArgs& a, const StreamShape& sp, cudaStream_t s) {
    auto kernel = gemv_stream_kernel<TYPE, CH>;
    constexpr int smem = stream_stages<TYPE>() * (kStreamQs + kStreamMeta);
    // a per-device attribute: set on every launch
    TVARA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    static const int per_sm = [&] {  // resident CTAs per SM (the same on every B200)
        int n = 0;
        TVARA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kStreamThreads, smem));
        return n > 0 ? n : 1;
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(sp.groups, gemv_sm_count() * per_sm));
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TVARA_CUDA(cudaLaunchKernelEx(&cfg, kernel, a, sp));
    TVARA_LAUNCHED();
    return true;
}

// Streamed single-token GEMV for the integer formats when the rows allow
// 16-byte bulk copies of whole units and headers (K a multiple of 256, at
// least 32 units per row); false when the caller should use another kernel.
template <int TYPE>
bool launch_gemv_stream(const GemmArgs& a, cudaStream_t s) {
    constexpr int E = Unit<TYPE>::kElems;
    const int units = a.w.cols / E;
    if (a.tokens != 1 || a.w.cols % 256 || units < 32 || a.w.rows < 1) return false;
    if ((reinterpret_cast<std::uintptr_t>(a.x) | reinterpret_cast<std::uintptr_t>(a.w.qs) |
         reinterpret_cast<std::uintptr_t>(a.w.meta) | a.w.qs_row | a.w.meta_row) & 15)
        return false;
    StreamShape sp;
    sp.kcu = 32;
    while (sp.kcu < 256 && sp.kcu * 2 <= units) sp.kcu *= 2;
    sp.rg = 1024 / sp.kcu;
    sp.chunks = (units + sp.kcu - 1) / sp.kcu;
    sp.groups = (a.w.rows + sp.rg - 1) / sp.rg;
    // x units held per lane: up to 2 (4-bit formats) or 4 (Q8_0) chunks of K
    switch (sp.chunks) {
        case 1: return launch_gemv_stream_ch<TYPE, 1>(a, sp, s);
        case 2: return launch_gemv_stream_ch<TYPE, 2>(a, sp, s);
        case 3: return TYPE == kQ8_0 && launch_gemv_stream_ch<TYPE, TYPE == kQ8_0 ? 3 : 1>(a, sp, s);
        case 4: return TYPE == kQ8_0 && launch_gemv_stream_ch<TYPE, TYPE == kQ8_0 ? 4 : 1>(a, sp, s);
    }
    return false;
}

template <int TYPE>
void dispatch_tokens(const GemmArgs& a, cudaStream_t s) {
    const std::size_t smem1 = std::size_t(a.w.cols) * 4 + std::size_t(a.w.cols / Unit<TYPE>::kElems) * 4;
    if constexpr (TYPE == kQ4_0 || TYPE == kQ4_K || TYPE == kQ8_0) {
        if (launch_gemv_stream<TYPE>(a, s)) return;
    }
    if (a.tokens <= 1 && (reinterpret_cast<std::uintptr_t>(a.x) & 15) == 0 && a.w.rows >= kRows1 &&
        smem1 <= 100 * 1024) {
        const int rows_per_cta = kWarps * kRows1;
        TVARA_CUDA(cudaFuncSetAttribute(gemv1_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem1)));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((a.w.rows + rows_per_cta - 1) / rows_per_cta);
        cfg.blockDim = dim3(kWarps * 32);
        cfg.dynamicSmemBytes = smem1;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        TVARA_CUDA(cudaLaunchKernelEx(&cfg, gemv1_kernel<TYPE>, a));
        TVARA_LAUNCHED();
    } else if (a.tokens <= 1) {
        run_gemv<TYPE, 8, 1>(a, s);  // unaligned activations or < 4 rows: staged through shared memory
    } else if (a.tokens <= 2) {
        run_gemv<TYPE, 4, 2>(a, s);
    } else {
        run_gemv<TYPE, 4, 4>(a, s);
    }
}

}  // namespace

void launch_gemv(const GemmArgs& a, cudaStream_t s) {
    if (a.tokens <= 0) return;
    if (a.epilogue == kSwiGLU && (a.w.rows % 2)) throw std::invalid_argument("SwiGLU needs paired rows");
    switch (a.w.type) {
        case kQ8_0: dispatch_tokens<kQ8_0>(a, s); break;
        case kQ4_0: dispatch_tokens<kQ4_0>(a, s); break;
        case kQ4_K: dispatch_tokens<kQ4_K>(a, s); break;
        case kF16: dispatch_tokens<kF16>(a, s); break;
        case kF32: dispatch_tokens<kF32>(a, s); break;
        default: throw std::invalid_argument("unsupported projection type");
    }
}

void launch_dequantize(int type, const void* blocks, std::size_t nblocks, float* out, cudaStream_t s) {
    std::size_t per = 0, bytes = 0;
    if (!block_shape(type, per, bytes)) throw std::invalid_argument("unsupported quantized type");
    const std::size_t total = nblocks * per;
    if (!total) return;
    const int grid = int(std::min<std::size_t>((total + 255) / 256, 148 * 32));
    dequant_kernel<<<grid, 256, 0, s>>>(type, static_cast<const unsigned char*>(blocks), nblocks, out);
    TVARA_LAUNCHED();
}

void launch_repack(int type, const void* gguf, int rows, int cols, std::uint8_t* qs, std::uint8_t* meta,
                   cudaStream_t s) {
    if (type == kF32 || type == kF16) {
        TVARA_CUDA(cudaMemcpyAsync(qs, gguf, std::size_t(rows) * qs_row_bytes(type, cols), cudaMemcpyDeviceToDevice, s));
        return;
    }
    const int per = type == kQ4_K ? 256 : 32;
    const std::size_t total = std::size_t(rows) * (cols / per);
    const int grid = int(std::min<std::size_t>((total + 255) / 256, 148 * 32));
    repack_kernel<<<grid, 256, 0, s>>>(type, static_cast<const unsigned char*>(gguf), rows, cols, qs, meta);
    TVARA_LAUNCHED();
}

void launch_planes(const DeviceMatrix& w, std::uint16_t* hi, std::uint16_t* lo, cudaStream_t s) {
    if (!w.row_shift || w.cols % 2) throw std::invalid_argument("planes need row shifts and an even width");
    planes_kernel<<<148 * 8, 256, 0, s>>>(w, reinterpret_cast<unsigned*>(hi), reinterpret_cast<unsigned*>(lo));
    TVARA_LAUNCHED();
}

std::size_t q4k_planes_bytes(int rows, int cols) {
    return std::size_t(rows) * cols * 2 + std::size_t(rows) * (cols / 32) * 4 + std::size_t(rows) * (cols / 256) * 4 +
           std::size_t(rows) + 5 * 256;
}

void launch_q4k_planes(DeviceMatrix& w, void* storage, cudaStream_t s) {
    if (w.type != kQ4_K || w.cols % 256) throw std::invalid_argument("Q4_K planes need Q4_K rows");
    auto* at = static_cast<unsigned char*>(storage);
    auto take = [&](std::size_t bytes) {
        unsigned char* p = at;
        at += (bytes + 255) & ~std::size_t(255);
        return p;
    };
    auto* qplane = reinterpret_cast<std::uint16_t*>(take(std::size_t(w.rows) * w.cols * 2));
    auto* min_hi = reinterpret_cast<std::uint16_t*>(take(std::size_t(w.rows) * (w.cols / 32) * 2));
    auto* min_lo = reinterpret_cast<std::uint16_t*>(take(std::size_t(w.rows) * (w.cols / 32) * 2));
    auto* qscale = reinterpret_cast<float*>(take(std::size_t(w.rows) * (w.cols / 256) * 4));
    auto* shift = reinterpret_cast<signed char*>(take(std::size_t(w.rows)));
    q4k_min_shift_kernel<<<(w.rows + 7) / 8, 256, 0, s>>>(w, shift);
    TVARA_LAUNCHED();
    q4k_planes_kernel<<<148 * 8, 256, 0, s>>>(w, reinterpret_cast<unsigned*>(qplane), qscale, min_hi, min_lo, shift);
    TVARA_LAUNCHED();
    w.qplane = qplane;
    w.qscale = qscale;
    w.qmin_hi = min_hi;
    w.qmin_lo = min_lo;
    w.qmin_shift = shift;
}

std::size_t q4k_packed_form_bytes(int rows, int cols) {
    return std::size_t(rows) * (cols / 32) * 5 + std::size_t(rows) * (cols / 256) * 4 + std::size_t(rows) + 5 * 256;
}

void launch_q4k_packed_form(DeviceMatrix& w, void* storage, cudaStream_t s) {
    if (w.type != kQ4_K || w.cols % 256) throw std::invalid_argument("the packed Q4_K form needs Q4_K rows");
    auto* at = static_cast<unsigned char*>(storage);
    auto take = [&](std::size_t bytes) {
        unsigned char* p = at;
        at += (bytes + 255) & ~std::size_t(255);
        return p;
    };
    const std::size_t units = std::size_t(w.rows) * (w.cols / 32);
    auto* qsc = take(units);
    auto* min_hi = reinterpret_cast<std::uint16_t*>(take(units * 2));
    auto* min_lo = reinterpret_cast<std::uint16_t*>(take(units * 2));
    auto* qscale = reinterpret_cast<float*>(take(std::size_t(w.rows) * (w.cols / 256) * 4));
    auto* shift = reinterpret_cast<signed char*>(take(std::size_t(w.rows)));
    q4k_min_shift_kernel<<<(w.rows + 7) / 8, 256, 0, s>>>(w, shift);
    TVARA_LAUNCHED();
    q4k_side_kernel<<<148 * 8, 256, 0, s>>>(w, qsc, qscale, min_hi, min_lo, shift);
    TVARA_LAUNCHED();
    w.qplane = nullptr;
    w.qsc = qsc;
    w.qscale = qscale;
    w.qmin_hi = min_hi;
    w.qmin_lo = min_lo;
    w.qmin_shift = shift;
}

void launch_finite_check(const DeviceMatrix& w, int* flag, cudaStream_t s) {
    finite_kernel<<<148 * 8, 256, 0, s>>>(w, flag);
    TVARA_LAUNCHED();
}

void launch_row_shift(const DeviceMatrix& w, signed char* out, cudaStream_t s) {
    if (w.rows <= 0) return;
    row_shift_kernel<<<(w.rows + 7) / 8, 256, 0, s>>>(w, out);
    TVARA_LAUNCHED();
}

void launch_embed(const DeviceMatrix& emb, const int* tokens, int n, float* x, int ldx, cudaStream_t s, int* ids,
                  const int* blk, const int* slot, int tpb) {
    if (n <= 0) return;
    embed_kernel<<<n, 256, 0, s>>>(emb, tokens, x, ldx, ids, blk, slot, tpb);
    TVARA_LAUNCHED();
}

}  // namespace tvara
