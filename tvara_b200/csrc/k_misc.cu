// RMSNorm, RoPE + paged-KV write, argmax and block copies.
#include <cfloat>

#include "kernels.cuh"

namespace tvara {
namespace {

// RMSNorm of core/include/tvara/model.hpp:57-65: sum of squares in double,
// inverse = float(1/sqrt(sum/n + eps)), out = (x*inverse)*w rounded twice.
template <bool HALF>
__global__ void rmsnorm_kernel(const float* x, int ldx, const int* rows, int dim, const float* w, float eps,
                               float* out, int ldo, __half* outh) {
    const int i = blockIdx.x;
    const long long r = rows ? rows[i] : i;
    const float* xr = x + r * ldx;
    double s = 0.0;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        const double v = xr[k];
        s += v * v;
    }
    __shared__ double part[32];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float inv = float(1.0 / sqrt(part[0] / double(dim) + double(eps)));
    float* o = out + (long long)i * ldo;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(xr[k], inv), w[k]);
        o[k] = v;
        if (HALF) outh[(long long)i * dim + k] = __float2half_rn(v);
    }
}

// RoPE of model.hpp:67-76 with the cos/sin table the host built from the
// reference's own float expression; pairs are (i, i+d/2) for the split layout
// and (2i, 2i+1) interleaved.  The rotation keeps the reference's two
// roundings per term (no contraction).  One CTA per token.
__global__ void rope_kv_kernel(RopeArgs a) {
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
            if (a.kv_f16) {
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
    if (!ok) return;
    const float* v = row + (a.hq + a.hkv) * d;
    for (int e = threadIdx.x; e < a.hkv * d; e += blockDim.x) {
        const int h = e / d, i = e % d;
        const long long off = base + a.kind_stride + ((long long)h * a.tpb + slot) * d + i;
        if (a.kv_f16) static_cast<__half*>(a.kv)[off] = __float2half_rn(v[e]);
        else static_cast<float*>(a.kv)[off] = v[e];
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

__global__ void swiglu_kernel(float* g, const float* u, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float x = g[i];
        const float small = expf(-fabsf(x));
        const float sig = x >= 0.f ? 1.f / (1.f + small) : small / (1.f + small);
        g[i] = __fmul_rn(x, __fmul_rn(sig, u[i]));
    }
}

__global__ void block_copy_kernel(uint4* kv, long long block_vec, const int2* pairs) {
    const int2 p = pairs[blockIdx.y];
    const uint4* src = kv + (long long)p.x * block_vec;
    uint4* dst = kv + (long long)p.y * block_vec;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < block_vec; i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace

void launch_rmsnorm(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps, float* out,
                    int ldo, cudaStream_t s) {
    if (n <= 0) return;
    rmsnorm_kernel<false><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, nullptr);
    TVARA_LAUNCHED();
}

void launch_rmsnorm_h(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps, float* out,
                      int ldo, __half* outh, cudaStream_t s) {
    if (n <= 0) return;
    rmsnorm_kernel<true><<<n, 256, 0, s>>>(x, ldx, rows, dim, w, eps, out, ldo, outh);
    TVARA_LAUNCHED();
}

void launch_rope_kv(const RopeArgs& a, cudaStream_t s) {
    if (a.tokens <= 0) return;
    rope_kv_kernel<<<a.tokens, 256, 0, s>>>(a);
    TVARA_LAUNCHED();
}

void launch_argmax(const float* logits, int rows, int vocab, unsigned* out, bool finite_check, cudaStream_t s) {
    if (rows <= 0) return;
    argmax_kernel<<<rows, 512, 0, s>>>(logits, vocab, out, int(finite_check));
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

}  // namespace tvara
