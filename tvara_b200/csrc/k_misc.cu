// RMSNorm, RoPE + paged-KV write, argmax and block copies.
#include <cfloat>

#include <cstdint>
#include <stdexcept>

#include "kernels.cuh"
#include "split.cuh"

namespace tvara {
namespace {

// RMSNorm of core/include/tvara/model.hpp:57-65: sum of squares in double,
// inverse = float(1/sqrt(sum/n + eps)), out = (x*inverse)*w rounded twice.
// One CTA (256 threads) per row;
// the row is loaded once as float4 and kept in registers (V per thread) for
// the output pass.  With SPLIT the normalised row is also written as the
// exact hi/lo FP16 split with its per-row power-of-two scale (max |v| in
// [2^14, 2^15)) -- the tensor-core projection's input format.
template <int V, bool SPLIT>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, int ldx, const int* rows, int dim, const float* w,
                                                      float eps, float* out, int ldo, __half* hi, __half* lo,
                                                      int* shift, __half* shi, __half* slo) {
    const int i = blockIdx.x;
    const long long r = rows ? rows[i] : i;
    const float4* xr = reinterpret_cast<const float4*>(x + r * ldx);
    const int n4 = dim / 4;
    float4 v[V];
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int k = threadIdx.x + j * 256;
        v[j] = k < n4 ? xr[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += double(v[j].x) * v[j].x + double(v[j].y) * v[j].y + double(v[j].z) * v[j].z + double(v[j].w) * v[j].w;
    }
    __shared__ double part[8];
    __shared__ float pmax[8];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += part[k];
    const float inv = float(1.0 / sqrt(tot / double(dim) + double(eps)));
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int k = threadIdx.x + j * 256;
        if (k < n4) {
            const float4 g = w4[k];
            v[j] = make_float4(__fmul_rn(__fmul_rn(v[j].x, inv), g.x), __fmul_rn(__fmul_rn(v[j].y, inv), g.y),
                               __fmul_rn(__fmul_rn(v[j].z, inv), g.z), __fmul_rn(__fmul_rn(v[j].w, inv), g.w));
            if (out) reinterpret_cast<float4*>(out + (long long)i * ldo)[k] = v[j];
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
        }
    }
    if constexpr (SPLIT) {
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31) == 0) pmax[threadIdx.x >> 5] = m;
        __syncthreads();
        float mx = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) mx = fmaxf(mx, pmax[k]);
        int e = 0;
        if (mx > 0.f && isfinite(mx)) frexpf(mx, &e);
        const int sh = mx > 0.f ? max(-100, min(100, 15 - e)) : 0;
        if (threadIdx.x == 0) shift[i] = sh;
        const float f = __uint_as_float(unsigned(127 + sh) << 23);
        uint2* hrow = reinterpret_cast<uint2*>(hi + (long long)i * dim);
        uint2* lrow = reinterpret_cast<uint2*>(lo + (long long)i * dim);
        const float f32 = __uint_as_float(unsigned(127 + sh - 5) << 23);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int k = threadIdx.x + j * 256;
            if (k < n4) {
                uint2 h, l;
                split_exact(v[j].x * f, v[j].y * f, h.x, l.x);
                split_exact(v[j].z * f, v[j].w * f, h.y, l.y);
                hrow[k] = h;
                lrow[k] = l;
            }
            // the Q4_K min term's sub-block sums (v[j] is zero past the row)
            if (dim % 32 == 0)
                subblock_sum_split(v[j], k, k < n4, f32, shi + (long long)i * (dim / 32), slo + (long long)i * (dim / 32));
        }
    }
}

// One warp: the reference's int8 encode of a row of d floats
// (python/tvara/quantized_kv.py:21-30): scale = max|x| / 127 (1 for a zero
// row, the smallest positive float if that underflows), codes rint(x / scale)
// clipped to [-127, 127]; a non-finite row records error 3.
__device__ void encode_row_i8(const float* src, int d, signed char* dst, float* scale_out, int* err) {
    const int lane = threadIdx.x & 31;
    float mx = 0.f;
    int bad = 0;
    for (int i = lane; i < d; i += 32) {
        bad |= !isfinite(src[i]);
        mx = fmaxf(mx, fabsf(src[i]));
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad = __any_sync(0xffffffffu, bad);
    if (bad && lane == 0) atomicExch(err, 3);  // "Nonfinite KV input"
    float scale = mx > 0.f ? __fdiv_rn(mx, 127.f) : 1.f;
    if (scale == 0.f) scale = __int_as_float(1);
    for (int i = lane; i < d; i += 32)
        dst[i] = (signed char)int(fminf(fmaxf(rintf(__fdiv_rn(src[i], scale)), -127.f), 127.f));
    if (lane == 0) *scale_out = scale;
}

__global__ void kv_quantize_kernel(const float* rows, int n, int d, signed char* codes, float* scales, int* err) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r < n) encode_row_i8(rows + (long long)r * d, d, codes + (long long)r * d, scales + r, err);
}

// RoPE of model.hpp:67-76 with the cos/sin table the host built from the
// reference's own float expression; pairs are (i, i+d/2) for the split layout
// and (2i, 2i+1) interleaved.  The rotation keeps the reference's two
// roundings per term (no contraction).  One CTA per token.
__global__ void rope_kv_kernel(RopeArgs a) {
    extern __shared__ float rkv[];  // int8 pools: the token's rotated K rows, then its V rows
    const int t = blockIdx.x;
    const int d = a.dim, half = d / 2;
    const long long pos = a.positions[t];
    const float* c = a.cosines + pos * half;
    const float* sn = a.sines + pos * half;
    const float* row = a.qkv + (long long)t * a.ldqkv;
    const int blk = a.slot_block[t], slot = a.slot_index[t];
    const bool ok = blk >= 0 && blk < a.max_blocks && slot >= 0 && slot < a.tpb;
    if (!ok && threadIdx.x == 0) atomicExch(a.err, 1);
    const long long base = (long long)blk * a.block_stride + a.layer_offset;
    const int qpairs = a.hq * half, kpairs = a.hkv * half;
    for (int p = threadIdx.x; p < qpairs + kpairs; p += blockDim.x) {
        const bool is_q = p < qpairs;
        const int pp = is_q ? p : p - qpairs;
        const int h = pp / half, i = pp % half;
        const float* src = row + (is_q ? 0 : a.hq * d) + h * d;
        const int ia = a.interleaved ? 2 * i : i, ib = a.interleaved ? 2 * i + 1 : i + half;
        const float left = src[ia], right = src[ib];
        const float ra = __fsub_rn(__fmul_rn(left, c[i]), __fmul_rn(right, sn[i]));
        const float rb = __fadd_rn(__fmul_rn(right, c[i]), __fmul_rn(left, sn[i]));
        if (is_q) {
            float* q = a.q + (long long)t * a.hq * d + h * d;
            q[ia] = ra;
            q[ib] = rb;
        } else if (ok) {
            const long long off = base + ((long long)h * a.tpb + slot) * d;
            if (a.kv_i8) {
                rkv[h * d + ia] = ra;
                rkv[h * d + ib] = rb;
            } else if (a.kv_f16) {
                __half* kv = static_cast<__half*>(a.kv);
                kv[off + ia] = __float2half_rn(ra);
                kv[off + ib] = __float2half_rn(rb);
            } else {
                float* kv = static_cast<float*>(a.kv);
                kv[off + ia] = ra;
                kv[off + ib] = rb;
            }
        }
    }
    if (!ok) return;  // uniform over the block
    const float* v = row + (a.hq + a.hkv) * d;
    for (int e = threadIdx.x; e < a.hkv * d; e += blockDim.x) {
        const int h = e / d, i = e % d;
        const long long off = base + a.kind_stride + ((long long)h * a.tpb + slot) * d + i;
        if (a.kv_i8) rkv[a.hkv * d + e] = v[e];
        else if (a.kv_f16) static_cast<__half*>(a.kv)[off] = __float2half_rn(v[e]);
        else static_cast<float*>(a.kv)[off] = v[e];
    }
    if (!a.kv_i8) return;
    // int8 rows, one warp per (kind, head)
    __syncthreads();
    for (int r = threadIdx.x >> 5; r < 2 * a.hkv; r += blockDim.x >> 5) {
        const int kind = r < a.hkv ? 0 : 1, h = r % a.hkv;
        const long long off = base + kind * a.kind_stride + ((long long)h * a.tpb + slot) * d;
        encode_row_i8(rkv + r * d, d, static_cast<signed char*>(a.kv) + off, a.kv_scales + off / d, a.err);
    }
}

// First index of the maximum; NaN ranks above every number (numpy.argmax).
// With finite_check, a row holding any NaN or infinity reports 0xFFFFFFFF.
__global__ void argmax_kernel(const float* logits, int vocab, unsigned* out, int finite_check) {
    const float* row = logits + (long long)blockIdx.x * vocab;
    float best = -INFINITY;
    int idx = INT_MAX;
    bool nan = false;
    bool bad = false;
    for (int k = threadIdx.x; k < vocab; k += blockDim.x) {
        const float v = row[k];
        bad |= !isfinite(v);
        if (isnan(v)) {
            if (!nan || k < idx) {
                nan = true;
                idx = k;
            }
        } else if (!nan && (v > best || (v == best && k < idx))) {
            best = v;
            idx = k;
        }
    }
    __shared__ float sb[32];
    __shared__ int si[32];
    __shared__ int sn[32];
    const int any_bad = __syncthreads_or(bad);
    for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        const int on = __shfl_xor_sync(0xffffffffu, int(nan), o);
        if (on && (!nan || oi < idx)) {
            nan = true;
            idx = oi;
        } else if (!on && !nan && (ob > best || (ob == best && oi < idx))) {
            best = ob;
            idx = oi;
        }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sb[w] = best;
        si[w] = idx;
        sn[w] = nan;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int j = 1; j < int(blockDim.x >> 5); ++j) {
            if (sn[j] && (!nan || si[j] < idx)) {
                nan = true;
                idx = si[j];
            } else if (!sn[j] && !nan && (sb[j] > best || (sb[j] == best && si[j] < idx))) {
                best = sb[j];
                idx = si[j];
            }
        }
        out[blockIdx.x] = finite_check && any_bad ? 0xFFFFFFFFu : unsigned(idx == INT_MAX ? 0 : idx);
    }
}

// Argmax over a vocabulary split across ranks: each rank reduces its slice
// of columns [col0, col0 + cols) of every row to one record (the slice's
// best value and global index with numpy.argmax's rules -- the first NaN
// ranks above every number -- and whether it saw a non-finite value); the
// records of all ranks (gathered [rank][row]) merge to the row's answer.
struct ArgmaxPart {
    float best;
    int idx;   // global column; INT_MAX when the slice is empty
    int nan;   // idx is the slice's first NaN
    int bad;   // a NaN or an infinity in the slice
};

__device__ __forceinline__ void argmax_take(float& best, int& idx, bool& nan, float ob, int oi, bool on) {
    if (on && (!nan || oi < idx)) {
        nan = true;
        idx = oi;
    } else if (!on && !nan && (ob > best || (ob == best && oi < idx))) {
        best = ob;
        idx = oi;
    }
}

__global__ void argmax_part_kernel(const float* logits, int ld, int cols, int col0, ArgmaxPart* out) {
    const float* row = logits + (long long)blockIdx.x * ld;
    float best = -INFINITY;
    int idx = INT_MAX;
    bool nan = false, bad = false;
    for (int k = threadIdx.x; k < cols; k += blockDim.x) {
        const float v = row[k];
        bad |= !isfinite(v);
        argmax_take(best, idx, nan, v, col0 + k, isnan(v));
    }
    __shared__ float sb[32];
    __shared__ int si[32], sn[32];
    const int any_bad = __syncthreads_or(bad);
    for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        const int on = __shfl_xor_sync(0xffffffffu, int(nan), o);
        argmax_take(best, idx, nan, ob, oi, on);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sb[w] = best;
        si[w] = idx;
        sn[w] = nan;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int j = 1; j < int(blockDim.x >> 5); ++j) argmax_take(best, idx, nan, sb[j], si[j], sn[j]);
        out[blockIdx.x] = ArgmaxPart{best, idx, int(nan), any_bad};
    }
}

__global__ void argmax_merge_kernel(const ArgmaxPart* parts, int rows, int ranks, unsigned* out, int finite_check) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float best = -INFINITY;
    int idx = INT_MAX;
    bool nan = false, bad = false;
    for (int k = 0; k < ranks; ++k) {
        const ArgmaxPart p = parts[(long long)k * rows + r];
        bad |= p.bad != 0;
        if (p.idx != INT_MAX) argmax_take(best, idx, nan, p.best, p.idx, p.nan != 0);
    }
    out[r] = finite_check && bad ? 0xFFFFFFFFu : unsigned(idx == INT_MAX ? 0 : idx);
}

__global__ void swiglu_kernel(float* g, const float* u, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float x = g[i];
        const float small = expf(-fabsf(x));
        const float sig = x >= 0.f ? 1.f / (1.f + small) : small / (1.f + small);
        g[i] = __fmul_rn(x, __fmul_rn(sig, u[i]));
    }
}

// Token ids of copied blocks (any block size).
__global__ void id_copy_kernel(int* ids, int per_block, const int2* pairs) {
    const int2 p = pairs[blockIdx.x];
    for (int i = threadIdx.x; i < per_block; i += blockDim.x)
        ids[(long long)p.y * per_block + i] = ids[(long long)p.x * per_block + i];
}

__global__ void block_copy_kernel(uint4* kv, long long block_vec, const int2* pairs) {
    const int2 p = pairs[blockIdx.y];
    const uint4* src = kv + (long long)p.x * block_vec;
    uint4* dst = kv + (long long)p.y * block_vec;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < block_vec; i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace

namespace {
template <bool SPLIT>
void run_rmsnorm(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps, float* out,
                 int ldo, __half* hi, __half* lo, int* shift, __half* shi, __half* slo, cudaStream_t s) {
    if (n <= 0) return;
    if (dim % 4 || (reinterpret_cast<std::uintptr_t>(x) & 15) || ldx % 4 || (out && ((reinterpret_cast<std::uintptr_t>(out) & 15) || ldo % 4)))
        throw std::invalid_argument("RMSNorm rows must be 16-byte aligned");
    const int v = (dim / 4 + 255) / 256;
    switch (v) {
        case 1: rmsnorm_kernel<1, SPLIT><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, hi, lo, shift, shi, slo); break;
        case 2: rmsnorm_kernel<2, SPLIT><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, hi, lo, shift, shi, slo); break;
        case 3:
        case 4: rmsnorm_kernel<4, SPLIT><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, hi, lo, shift, shi, slo); break;
        case 5:
        case 6:
        case 7:
        case 8: rmsnorm_kernel<8, SPLIT><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, hi, lo, shift, shi, slo); break;
        default: throw std::invalid_argument("RMSNorm width above 8192");
    }
    TVARA_LAUNCHED();
}
}  // namespace

void launch_rmsnorm(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps, float* out,
                    int ldo, cudaStream_t s) {
    run_rmsnorm<false>(x, ldx, rows, n, dim, w, eps, out, ldo, nullptr, nullptr, nullptr, nullptr, nullptr, s);
}

void launch_rmsnorm_split(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps,
                          float* out, int ldo, void* tc_workspace, std::size_t tc_workspace_bytes, cudaStream_t s) {
    __half *hi = nullptr, *lo = nullptr, *shi = nullptr, *slo = nullptr;
    int* shift = nullptr;
    gemm_tc_split_buffers(tc_workspace, tc_workspace_bytes, n, dim, hi, lo, shift, &shi, &slo);
    run_rmsnorm<true>(x, ldx, rows, n, dim, w, eps, out, ldo, hi, lo, shift, shi, slo, s);
}

void launch_kv_quantize(const float* rows, int n, int d, signed char* codes, float* scales, int* err, cudaStream_t s) {
    if (n <= 0) return;
    kv_quantize_kernel<<<(n + 7) / 8, 256, 0, s>>>(rows, n, d, codes, scales, err);
    TVARA_LAUNCHED();
}

std::size_t rope_kv_smem(const RopeArgs& a) {
    return a.kv_i8 ? std::size_t(2) * a.hkv * a.dim * sizeof(float) : 0;
}

void launch_rope_kv(const RopeArgs& a, cudaStream_t s) {
    if (a.tokens <= 0) return;
    if (a.kv_i8 && (!a.kv_scales || rope_kv_smem(a) > 48 * 1024))
        throw std::invalid_argument("int8 KV: scales missing or KV heads x head_dim above 6144");
    rope_kv_kernel<<<a.tokens, 256, rope_kv_smem(a), s>>>(a);
    TVARA_LAUNCHED();
}

void launch_argmax(const float* logits, int rows, int vocab, unsigned* out, bool finite_check, cudaStream_t s) {
    if (rows <= 0) return;
    argmax_kernel<<<rows, 512, 0, s>>>(logits, vocab, out, int(finite_check));
    TVARA_LAUNCHED();
}

std::size_t argmax_part_bytes() { return sizeof(ArgmaxPart); }

void launch_argmax_part(const float* logits, int rows, int ld, int cols, int col0, void* parts, cudaStream_t s) {
    if (rows <= 0) return;
    argmax_part_kernel<<<rows, 512, 0, s>>>(logits, ld, cols, col0, static_cast<ArgmaxPart*>(parts));
    TVARA_LAUNCHED();
}

void launch_argmax_merge(const void* parts, int rows, int ranks, unsigned* out, bool finite_check, cudaStream_t s) {
    if (rows <= 0) return;
    argmax_merge_kernel<<<(rows + 127) / 128, 128, 0, s>>>(static_cast<const ArgmaxPart*>(parts), rows, ranks, out,
                                                           int(finite_check));
    TVARA_LAUNCHED();
}

void launch_swiglu(float* g, const float* u, long long n, cudaStream_t s) {
    if (n <= 0) return;
    swiglu_kernel<<<int(std::min<long long>((n + 255) / 256, 148 * 16)), 256, 0, s>>>(g, u, n);
    TVARA_LAUNCHED();
}

void launch_block_copy(void* kv, long long block_bytes, const int2* pairs, int n, cudaStream_t s) {
    if (n <= 0) return;
    if (block_bytes % 16) throw std::invalid_argument("KV block size must be a multiple of 16 bytes");
    block_copy_kernel<<<dim3(64, n), 256, 0, s>>>(static_cast<uint4*>(kv), block_bytes / 16, pairs);
    TVARA_LAUNCHED();
}

void launch_id_copy(int* ids, int per_block, const int2* pairs, int n, cudaStream_t s) {
    if (n <= 0) return;
    id_copy_kernel<<<n, 128, 0, s>>>(ids, per_block, pairs);
    TVARA_LAUNCHED();
}

}  // namespace tvara
