// Paged GQA attention over ragged per-sequence block lists (decode and
// chunked prefill share it: every query token attends to positions
// [0, pos] of its sequence, its own K/V already written to the pool).
//
// Semantics follow core/include/tvara/attention.hpp:57-83: query head h
// reads KV head h/(Hq/Hkv), score = q.k/sqrt(d), softmax over the visible
// positions, weighted sum of V.  The reference accumulates in double; here
// scores and the running softmax are F32 with an online (max-rescaled)
// update, which stays within ~1e-6 relative of it.
//
// Pool layout (elements): block b, layer l, kind (0 = K, 1 = V), KV head h,
// slot s, element e at b*block_stride + l*layer_stride + kind*kind_stride +
// (h*tpb + s)*d + e, so one head's slots of a block are one contiguous run.
//
// CTA = 4 warps on one (work item, KV head).  A work item is a position range
// of one token; long contexts are split over several items whose partial
// (max, sum, weighted V) are merged by combine_kernel.
#include <cfloat>

#include "kernels.cuh"

namespace tvara {
namespace {

constexpr int kAttnWarps = 4;

template <typename KV, int VEC>
__device__ __forceinline__ void load_vec(const KV* p, bool ok, float (&out)[VEC]) {
    if constexpr (sizeof(KV) == 4) {
#pragma unroll
        for (int j = 0; j < VEC; j += 4) {
            float4 v = ok ? __ldg(reinterpret_cast<const float4*>(p + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
            out[j] = v.x;
            out[j + 1] = v.y;
            out[j + 2] = v.z;
            out[j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < VEC; j += 8) {
            uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(p + j)) : make_uint4(0, 0, 0, 0);
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h[i]);
                out[j + 2 * i] = f.x;
                out[j + 2 * i + 1] = f.y;
            }
        }
    }
}

template <int D, typename KV, int G>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(AttnArgs a) {
    constexpr int ES = sizeof(KV);
    constexpr int LPS = (D * ES / 16) < 32 ? (D * ES / 16) : 32;  // lanes per slot
    constexpr int VEC = D / LPS;                                // elements per lane
    constexpr int SPL = 32 / LPS;                               // slots per warp pass
    constexpr int NIT = (64 / (VEC * ES)) > 0 ? (64 / (VEC * ES)) : 1;  // passes per chunk
    constexpr int CH = SPL * NIT;                               // slots per chunk

    const int4 wk = a.work[blockIdx.x];
    const int part = a.work_part[blockIdx.x];
    const int t = wk.x, toff = wk.y, p0 = wk.z, p1 = wk.w;
    const int h = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane % LPS, grp = lane / LPS;
    const float scale = rsqrtf(float(D));

    float q[G][VEC];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float* qp = a.q + (long long)t * a.hq * D + (h * G + g) * D + sub * VEC;
#pragma unroll
        for (int j = 0; j < VEC; ++j) q[g][j] = qp[j] * scale;
    }
    float acc[G][VEC], l[G], m[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        l[g] = 0.f;
        m[g] = -INFINITY;
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[g][j] = 0.f;
    }

    const KV* pool = static_cast<const KV*>(a.kv);
    const int tpb = a.tpb;
    const int b0 = p0 / tpb, b1 = (p1 - 1) / tpb;
    for (int bi = b0 + warp; bi <= b1; bi += kAttnWarps) {
        const int pb = a.tables[toff + bi];
        if (pb < 0 || pb >= a.max_blocks) {
            if (lane == 0) atomicExch(a.err, 2);
            continue;
        }
        const int s_lo = bi == b0 ? p0 - bi * tpb : 0;
        const int s_hi = min(tpb, p1 - bi * tpb);
        const KV* kb = pool + (long long)pb * a.block_stride + a.layer_offset + (long long)h * tpb * D;
        const KV* vb = kb + a.kind_stride;
        for (int c0 = s_lo; c0 < s_hi; c0 += CH) {
            float kv[NIT][VEC];
            bool valid[NIT];
#pragma unroll
            for (int it = 0; it < NIT; ++it) {
                const int s = c0 + it * SPL + grp;
                valid[it] = s < s_hi;
                load_vec<KV, VEC>(kb + (long long)s * D + sub * VEC, valid[it], kv[it]);
            }
            float sc[NIT][G];
            float cmax[G];
#pragma unroll
            for (int g = 0; g < G; ++g) cmax[g] = -INFINITY;
#pragma unroll
            for (int it = 0; it < NIT; ++it) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < VEC; ++j) d = fmaf(q[g][j], kv[it][j], d);
#pragma unroll
                    for (int o = LPS / 2; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    sc[it][g] = valid[it] ? d : -INFINITY;
                    cmax[g] = fmaxf(cmax[g], sc[it][g]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
#pragma unroll
                for (int o = LPS; o < 32; o <<= 1) cmax[g] = fmaxf(cmax[g], __shfl_xor_sync(0xffffffffu, cmax[g], o));
                const float mn = fmaxf(m[g], cmax[g]);
                const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - mn);
                m[g] = mn;
                l[g] *= alpha;
#pragma unroll
                for (int j = 0; j < VEC; ++j) acc[g][j] *= alpha;
#pragma unroll
                for (int it = 0; it < NIT; ++it) {
                    sc[it][g] = valid[it] ? expf(sc[it][g] - mn) : 0.f;
                    l[g] += sc[it][g];
                }
            }
#pragma unroll
            for (int it = 0; it < NIT; ++it) {
                const int s = c0 + it * SPL + grp;
                load_vec<KV, VEC>(vb + (long long)s * D + sub * VEC, valid[it], kv[it]);
            }
#pragma unroll
            for (int it = 0; it < NIT; ++it)
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int j = 0; j < VEC; ++j) acc[g][j] = fmaf(sc[it][g], kv[it][j], acc[g][j]);
        }
    }
    // merge the slot groups of the warp (lanes with equal `sub`)
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = LPS; o < 32; o <<= 1) {
            l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
            for (int j = 0; j < VEC; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
        }
    }
    __shared__ float s_acc[kAttnWarps][G][D];
    __shared__ float s_m[kAttnWarps][G], s_l[kAttnWarps][G];
    if (lane < LPS) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < VEC; ++j) s_acc[warp][g][sub * VEC + j] = acc[g][j];
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            s_m[warp][g] = m[g];
            s_l[warp][g] = l[g];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, e = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w][g]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            if (s_m[w][g] == -INFINITY) continue;
            const float f = expf(s_m[w][g] - M);
            L = fmaf(s_l[w][g], f, L);
            A = fmaf(s_acc[w][g][e], f, A);
        }
        const int head = h * G + g;
        if (part < 0) {
            a.out[(long long)t * a.hq * D + head * D + e] = A / L;
        } else {
            float* pp = a.partial + ((long long)part * a.hq + head) * (D + 2);
            pp[e] = A;
            if (e == 0) {
                pp[D] = M;
                pp[D + 1] = L;
            }
        }
    }
}

// Merge split partials: out = sum_i A_i e^{M_i-M} / sum_i L_i e^{M_i-M}.
__global__ void combine_kernel(AttnArgs a) {
    const int4 c = a.combine[blockIdx.x];
    const int head = blockIdx.y, D = a.dim;
    const int t = c.x, first = c.y, n = c.z;
    for (int e = threadIdx.x; e < D; e += blockDim.x) {
        float M = -INFINITY;
        for (int i = 0; i < n; ++i) M = fmaxf(M, a.partial[((long long)(first + i) * a.hq + head) * (D + 2) + D]);
        float L = 0.f, A = 0.f;
        for (int i = 0; i < n; ++i) {
            const float* pp = a.partial + ((long long)(first + i) * a.hq + head) * (D + 2);
            if (pp[D] == -INFINITY) continue;
            const float f = expf(pp[D] - M);
            L = fmaf(pp[D + 1], f, L);
            A = fmaf(pp[e], f, A);
        }
        a.out[(long long)t * a.hq * D + head * D + e] = A / L;
    }
}

template <int D, typename KV>
void run_g(const AttnArgs& a, cudaStream_t s) {
    const int g = a.hq / a.hkv;
    dim3 grid(a.n_work, a.hkv);
    switch (g) {
#define TV_G(N) \
    case N: attn_kernel<D, KV, N><<<grid, kAttnWarps * 32, 0, s>>>(a); break;
        TV_G(1) TV_G(2) TV_G(3) TV_G(4) TV_G(5) TV_G(6) TV_G(7) TV_G(8)
#undef TV_G
        default: throw std::invalid_argument("unsupported query/KV head ratio (1..8)");
    }
}

template <typename KV>
void run_d(const AttnArgs& a, cudaStream_t s) {
    switch (a.dim) {
        case 32: run_g<32, KV>(a, s); break;
        case 64: run_g<64, KV>(a, s); break;
        case 128: run_g<128, KV>(a, s); break;
        case 256: run_g<256, KV>(a, s); break;
        case 16: run_g<16, KV>(a, s); break;
        default: throw std::invalid_argument("unsupported head_dim (16, 32, 64, 128, 256)");
    }
}

}  // namespace

void launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.n_work <= 0) return;
    if (a.kv_f16) run_d<__half>(a, s);
    else run_d<float>(a, s);
    TVARA_LAUNCHED();
    if (a.n_combine > 0) {
        combine_kernel<<<dim3(a.n_combine, a.hq), 128, 0, s>>>(a);
        TVARA_LAUNCHED();
    }
}

}  // namespace tvara
