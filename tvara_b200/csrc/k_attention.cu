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
#include <cstdint>
#include <string>
#include <type_traits>

#include "kernels.cuh"
#include "tma.cuh"

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
    } else if constexpr (sizeof(KV) == 1) {
        // int8 rows: the caller multiplies by the row's scale
#pragma unroll
        for (int j = 0; j < VEC; j += 16) {
            uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(p + j)) : make_uint4(0, 0, 0, 0);
            const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 16; ++i) out[j + i] = float(int((signed char)((w[i >> 2] >> (8 * (i & 3))) & 255u)));
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
                if constexpr (sizeof(KV) == 1) {
                    // decoded value = code * scale (quantized_kv.py:49-54), one F32 product
                    const float sc = valid[it] ? a.kv_scales[(kb - pool) / D + s] : 0.f;
#pragma unroll
                    for (int j = 0; j < VEC; ++j) kv[it][j] = __fmul_rn(kv[it][j], sc);
                }
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
                if constexpr (sizeof(KV) == 1) {
                    const float sc = valid[it] ? a.kv_scales[(vb - pool) / D + s] : 0.f;
#pragma unroll
                    for (int j = 0; j < VEC; ++j) kv[it][j] = __fmul_rn(kv[it][j], sc);
                }
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

// ---------------------------------------------------------------------------
// Pipelined variant: each warp owns a ring of shared-memory stages; its lane 0
// streams whole K and V chunks of the warp's KV blocks (one head's tpb x d run
// is contiguous in the pool) with cp.async.bulk onto a per-stage mbarrier, so
// several blocks per warp are in flight while the warp computes on one from
// shared memory.  Same arithmetic as attn_kernel.
constexpr int kRing = 2;                   // stages per warp
constexpr unsigned kAttnSpin = 1u << 26;   // bounded waits

__device__ __forceinline__ unsigned s_u32(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, std::uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     s_u32(dst)),
                 "l"(src), "r"(bytes), "r"(s_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool bar_try(std::uint64_t* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(s_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

template <typename KV, int VEC>
__device__ __forceinline__ void smem_vec(const KV* p, float (&out)[VEC]) {
    if constexpr (sizeof(KV) == 4) {
#pragma unroll
        for (int j = 0; j < VEC; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + j);
            out[j] = v.x;
            out[j + 1] = v.y;
            out[j + 2] = v.z;
            out[j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < VEC; j += 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(p + j);
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
__global__ void __launch_bounds__(kAttnWarps * 32) attn_pipe_kernel(AttnArgs a) {
    constexpr int ES = sizeof(KV);
    constexpr int LPS = (D * ES / 16) < 32 ? (D * ES / 16) : 32;
    constexpr int VEC = D / LPS;
    constexpr int SPL = 32 / LPS;
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int tpb = a.tpb;
    const int chunk = tpb * D * ES;  // bytes of one head's K (or V) run in a block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(att_smem) + warp * kRing;
    unsigned char* ring = att_smem + 128 + std::size_t(warp) * kRing * 2 * chunk;
    __shared__ float s_acc[kAttnWarps][G][D];
    __shared__ float s_m[kAttnWarps][G], s_l[kAttnWarps][G];

    const int4 wk = a.work[blockIdx.x];
    const int part = a.work_part[blockIdx.x];
    const int t = wk.x, toff = wk.y, p0 = wk.z, p1 = wk.w;
    const int h = blockIdx.y;
    const int sub = lane % LPS, grp = lane / LPS;
    const float scale = rsqrtf(float(D));
    const KV* pool = static_cast<const KV*>(a.kv);
    const int b0 = p0 / tpb, b1 = (p1 - 1) / tpb;
    // this warp's blocks: b0 + warp + 4*i, i < nblk
    const int nblk = b1 - b0 - warp >= 0 ? (b1 - b0 - warp) / kAttnWarps + 1 : 0;

    if (lane == 0) {
        for (int s = 0; s < kRing; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int i) {  // lane 0: start block i of this warp into stage i % kRing
        const int bi = b0 + warp + i * kAttnWarps;
        int pb = a.tables[toff + bi];
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;  // read something in range; the step reports the error
        }
        const KV* kb = pool + (long long)pb * a.block_stride + a.layer_offset + (long long)h * tpb * D;
        unsigned char* st = ring + std::size_t(i % kRing) * 2 * chunk;
        std::uint64_t* bar = &bars[i % kRing];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(bar)), "r"(2 * chunk) : "memory");
        bulk_g2s(st, kb, chunk, bar);
        bulk_g2s(st + chunk, kb + a.kind_stride, chunk, bar);
    };
    if (lane == 0)
        for (int i = 0; i < kRing && i < nblk; ++i) issue(i);

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
    bool failed = false;
    for (int i = 0; i < nblk; ++i) {
        const int bi = b0 + warp + i * kAttnWarps;
        const unsigned parity = (i / kRing) & 1;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[i % kRing], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const KV* ks = reinterpret_cast<const KV*>(ring + std::size_t(i % kRing) * 2 * chunk);
        const KV* vs = ks + tpb * D;
        const int s_hi = min(tpb, p1 - bi * tpb);
        constexpr int NI = 8;  // slot passes per softmax rescale
        for (int c0 = 0; c0 < s_hi; c0 += NI * SPL) {
            float sc[NI][G], cmax[G];
#pragma unroll
            for (int g = 0; g < G; ++g) cmax[g] = -INFINITY;
#pragma unroll
            for (int it = 0; it < NI; ++it) {
                const int s = c0 + it * SPL + grp;
                const bool valid = s < s_hi;
                float kv[VEC];
                if (valid) smem_vec<KV, VEC>(ks + s * D + sub * VEC, kv);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float d = 0.f;
                    if (valid) {
#pragma unroll
                        for (int j = 0; j < VEC; ++j) d = fmaf(q[g][j], kv[j], d);
                    }
#pragma unroll
                    for (int o = LPS / 2; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    sc[it][g] = valid ? d : -INFINITY;
                    cmax[g] = fmaxf(cmax[g], sc[it][g]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
#pragma unroll
                for (int o = LPS; o < 32; o <<= 1) cmax[g] = fmaxf(cmax[g], __shfl_xor_sync(0xffffffffu, cmax[g], o));
                const float mn = fmaxf(m[g], cmax[g]);
                const float alpha = m[g] == -INFINITY ? 0.f : __expf(m[g] - mn);
                m[g] = mn;
                l[g] *= alpha;
#pragma unroll
                for (int j = 0; j < VEC; ++j) acc[g][j] *= alpha;
#pragma unroll
                for (int it = 0; it < NI; ++it) {
                    sc[it][g] = sc[it][g] == -INFINITY ? 0.f : __expf(sc[it][g] - mn);
                    l[g] += sc[it][g];
                }
            }
#pragma unroll
            for (int it = 0; it < NI; ++it) {
                const int s = c0 + it * SPL + grp;
                if (s < s_hi) {
                    float kv[VEC];
                    smem_vec<KV, VEC>(vs + s * D + sub * VEC, kv);
#pragma unroll
                    for (int g = 0; g < G; ++g)
#pragma unroll
                        for (int j = 0; j < VEC; ++j) acc[g][j] = fmaf(sc[it][g], kv[j], acc[g][j]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + kRing < nblk) issue(i + kRing);
    }
    // every copy this warp started must land before the CTA exits
    if (lane == 0 && failed) {
        for (int i = 0; i < kRing && i < nblk; ++i)
            for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[i], 0) && !bar_try(&bars[i], 1); ++spin) {
            }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = LPS; o < 32; o <<= 1) {
            l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
            for (int j = 0; j < VEC; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
        }
    }
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
            const float f = __expf(s_m[w][g] - M);
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

// Packed F32x2 helpers (Blackwell fma.rn.f32x2).
__device__ __forceinline__ unsigned long long pk(float x, float y) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ float2 upk(unsigned long long r) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// VEC consecutive elements of a K or V slot from shared memory as packed pairs.
template <typename KV, int VEC>
__device__ __forceinline__ void smem_pairs(const KV* p, unsigned long long (&out)[VEC / 2]) {
    if constexpr (sizeof(KV) == 4) {
#pragma unroll
        for (int j = 0; j < VEC; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + j);
            out[j / 2] = pk(v.x, v.y);
            out[j / 2 + 1] = pk(v.z, v.w);
        }
    } else {
#pragma unroll
        for (int j = 0; j < VEC; j += 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(p + j);
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h[i]);
                out[j / 2 + i] = pk(f.x, f.y);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Per-warp ring (as attn_pipe_kernel) with a transposing score reduction, for
// G a power of two no larger than the lanes per slot: the G partial dots of a
// lane are reduced across the slot's LPS lanes in log2(LPS) + G - 1 shuffles
// (instead of G*log2(LPS)), after which each lane owns the score of one head
// (its softmax state too, one exponential per lane); the probabilities are
// broadcast back for the V pass.  Dots and the V accumulation use the packed
// F32x2 FMA.
template <int D, typename KV, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 3) attn_xpose_kernel(AttnArgs a) {
    constexpr int ES = sizeof(KV);
    constexpr int LPS = (D * ES / 16) < 32 ? (D * ES / 16) : 32;
    constexpr int VEC = D / LPS;
    constexpr int SPL = 32 / LPS;
    constexpr int NI = 8;
    constexpr int HL = LPS / G;  // lanes holding one head's score within a slot group
    static_assert((G & (G - 1)) == 0 && G <= LPS && VEC % 2 == 0, "transposing layout");
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int tpb = a.tpb;
    const int chunk = tpb * D * ES;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(att_smem) + warp * kRing;
    unsigned char* ring = att_smem + 128 + std::size_t(warp) * kRing * 2 * chunk;
    __shared__ float s_acc[kAttnWarps][G][D];
    __shared__ float s_m[kAttnWarps][G], s_l[kAttnWarps][G];

    const int4 wk = a.work[blockIdx.x];
    const int part = a.work_part[blockIdx.x];
    const int t = wk.x, toff = wk.y, p0 = wk.z, p1 = wk.w;
    const int h = blockIdx.y;
    const int sub = lane % LPS, grp = lane / LPS;
    const int mine = sub / HL;  // the head whose score this lane ends up holding
    const int gbase = lane - sub;
    const KV* pool = static_cast<const KV*>(a.kv);
    const int b0 = p0 / tpb, b1 = (p1 - 1) / tpb;
    const int nblk = b1 - b0 - warp >= 0 ? (b1 - b0 - warp) / kAttnWarps + 1 : 0;

    if (lane == 0) {
        for (int s = 0; s < kRing; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int i) {
        const int bi = b0 + warp + i * kAttnWarps;
        int pb = a.tables[toff + bi];
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;
        }
        const KV* kb = pool + (long long)pb * a.block_stride + a.layer_offset + (long long)h * tpb * D;
        unsigned char* st = ring + std::size_t(i % kRing) * 2 * chunk;
        std::uint64_t* bar = &bars[i % kRing];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(bar)), "r"(2 * chunk) : "memory");
        bulk_g2s(st, kb, chunk, bar);
        bulk_g2s(st + chunk, kb + a.kind_stride, chunk, bar);
    };
    if (lane == 0)
        for (int i = 0; i < kRing && i < nblk; ++i) issue(i);

    unsigned long long q2[G][VEC / 2], acc2[G][VEC / 2];
    {
        const float scale = rsqrtf(float(D));
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float* qp = a.q + (long long)t * a.hq * D + (h * G + g) * D + sub * VEC;
#pragma unroll
            for (int j = 0; j < VEC / 2; ++j) {
                q2[g][j] = pk(qp[2 * j] * scale, qp[2 * j + 1] * scale);
                acc2[g][j] = 0ull;
            }
        }
    }
    float l = 0.f, m = -INFINITY;  // softmax state of head `mine`
    bool failed = false;
    for (int i = 0; i < nblk; ++i) {
        const int bi = b0 + warp + i * kAttnWarps;
        const unsigned parity = (i / kRing) & 1;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[i % kRing], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const KV* ks = reinterpret_cast<const KV*>(ring + std::size_t(i % kRing) * 2 * chunk);
        const KV* vs = ks + tpb * D;
        const int s_hi = min(tpb, p1 - bi * tpb);
        for (int c0 = 0; c0 < s_hi; c0 += NI * SPL) {
            float sc[NI];
            float cmax = -INFINITY;
#pragma unroll
            for (int it = 0; it < NI; ++it) {
                const int s = c0 + it * SPL + grp;
                const bool valid = s < s_hi;
                float d[G];
                {
                    unsigned long long k2[VEC / 2];
                    if (valid) smem_pairs<KV, VEC>(ks + s * D + sub * VEC, k2);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        unsigned long long d2 = 0ull;
                        if (valid) {
#pragma unroll
                            for (int j = 0; j < VEC / 2; ++j) d2 = ffma2(q2[g][j], k2[j], d2);
                        }
                        const float2 f = upk(d2);
                        d[g] = f.x + f.y;
                    }
                }
                // transpose-reduce: halve the head set per exchange
#pragma unroll
                for (int n = G, o = LPS / 2; n > 1; n >>= 1, o >>= 1) {
                    const bool upper = (lane & o) != 0;
#pragma unroll
                    for (int g = 0; g < n / 2; ++g) {
                        const float send = upper ? d[g] : d[g + n / 2];
                        const float keep = upper ? d[g + n / 2] : d[g];
                        d[g] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                    }
                }
#pragma unroll
                for (int o = HL / 2; o; o >>= 1) d[0] += __shfl_xor_sync(0xffffffffu, d[0], o);
                sc[it] = valid ? d[0] : -INFINITY;
                cmax = fmaxf(cmax, sc[it]);
            }
#pragma unroll
            for (int o = LPS; o < 32; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
            const float mn = fmaxf(m, cmax);
            const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
            m = mn;
            l *= alpha;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float ag = __shfl_sync(0xffffffffu, alpha, gbase + g * HL);
                const unsigned long long a2 = pk(ag, ag);
#pragma unroll
                for (int j = 0; j < VEC / 2; ++j) acc2[g][j] = ffma2(acc2[g][j], a2, 0ull);
            }
#pragma unroll
            for (int it = 0; it < NI; ++it) {
                const int s = c0 + it * SPL + grp;
                const bool valid = s < s_hi;
                const float p = valid ? __expf(sc[it] - mn) : 0.f;
                l += p;
                unsigned long long v2[VEC / 2];
                if (valid) smem_pairs<KV, VEC>(vs + s * D + sub * VEC, v2);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg = __shfl_sync(0xffffffffu, p, gbase + g * HL);
                    if (valid) {
                        const unsigned long long p2 = pk(pg, pg);
#pragma unroll
                        for (int j = 0; j < VEC / 2; ++j) acc2[g][j] = ffma2(p2, v2[j], acc2[g][j]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + kRing < nblk) issue(i + kRing);
    }
    if (lane == 0 && failed) {
        for (int i = 0; i < kRing && i < nblk; ++i)
            for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[i], 0) && !bar_try(&bars[i], 1); ++spin) {
            }
    }
    // merge slot groups: acc for every head, l for this lane's head
#pragma unroll
    for (int o = LPS; o < 32; o <<= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < VEC / 2; ++j) {
                const float2 f = upk(acc2[g][j]);
                acc2[g][j] = pk(f.x + __shfl_xor_sync(0xffffffffu, f.x, o), f.y + __shfl_xor_sync(0xffffffffu, f.y, o));
            }
    }
    if (lane < LPS) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < VEC / 2; ++j) {
                const float2 f = upk(acc2[g][j]);
                s_acc[warp][g][sub * VEC + 2 * j] = f.x;
                s_acc[warp][g][sub * VEC + 2 * j + 1] = f.y;
            }
        if (sub % HL == 0) {
            s_m[warp][mine] = m;
            s_l[warp][mine] = l;
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
            const float f = __expf(s_m[w][g] - M);
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

// ---------------------------------------------------------------------------
// Tensor-core paged attention for F16 KV (head_dim 64 or 128, blocks of a
// multiple of 16 slots).  CTA = (work item, KV head), four warps; each warp
// streams its share of the blocks through a two-stage ring of TMA tensor
// copies (one box per 64 elements of head_dim, 128-byte swizzle, so the
// ldmatrix reads below are free of bank conflicts).  Per 16 positions a warp
// computes, with mma.m16n8k16 (F16 operands, F32 accumulation),
//   S^T [16 positions x 8 heads] = K [16 x D] . Q^T [D x 8]   and
//   O^T [D x 8 heads]           += V^T [D x 16] . P^T [16 x 8],
// the group's G <= 8 query heads being the N columns; P^T reaches the B
// operand layout by an in-register transpose (movmatrix) of the score tile.
// Q and P enter as exact hi + lo F16 pairs after a power-of-two scaling (Q
// per head so that |q| < 2^15, P by 2^11), so every product keeps about 22
// significant bits: the F32 attention of the kernels above to within
// rounding.  The softmax reference m of a head moves only when a score
// exceeds it by more than 4 ln 2 (a warp vote; then the reductions and the
// rescale of O), so P = e^(s - m) < 16 and most tiles skip both.
constexpr int kMmaRing = 2;
constexpr float kLazyMargin = 2.7725887f;  // 4 ln 2: softmax weights stay below 16

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// d += A b for one m16n8k16 tile (A row-major 16x16, b col-major 16x8).
__device__ __forceinline__ void mma16816(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Transpose of an 8x8 matrix of 16-bit values held one pair per lane.
__device__ __forceinline__ unsigned movmatrix_t(unsigned x) {
    unsigned y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// x, y as packed F16 pairs hi + lo with hi + lo == (x, y) to ~22 bits.
__device__ __forceinline__ void split_f16x2(float x, float y, unsigned& hi, unsigned& lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const unsigned*>(&h);
    lo = *reinterpret_cast<const unsigned*>(&l);
}
// 2^e for |e| <= 126, exact.
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(unsigned(127 + e) << 23); }

template <int D, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 3) attn_mma_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                      AttnArgs a) {
    constexpr int NB = D / 64;  // 128-byte boxes per slot row
    constexpr int KS = D / 16;  // k-steps of S^T, and m-tiles of O^T
    static_assert(D % 64 == 0 && G >= 1 && G <= 8, "tensor-core attention shape");
    // G <= 4: columns 4..7 of P^T carry the lo parts of heads 0..3, so one
    // value MMA per tile takes hi and lo (O^T columns 4..7 are added back at the end)
    constexpr bool kPackLo = G <= 4;
    extern __shared__ unsigned char att_raw[];
    __shared__ std::uint64_t bars[kAttnWarps][kMmaRing];
    __shared__ float s_m[kAttnWarps][8], s_l[kAttnWarps][8];
    const int tpb = a.tpb;
    const int box = tpb * 128;          // one box: tpb slots x 64 halves
    const int half_stage = NB * box;    // K (or V) of one block
    const int stage = 2 * half_stage;
    unsigned char* smem = att_raw + ((1024u - (s_u32(att_raw) & 1023u)) & 1023u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned char* ring = smem + std::size_t(warp) * kMmaRing * stage;
    const unsigned ring_s = s_u32(ring);

    const int4 wk = a.work[blockIdx.x];
    const int part = a.work_part[blockIdx.x];
    const int t = wk.x, toff = wk.y, p0 = wk.z, p1 = wk.w;
    const int h = blockIdx.y;
    const int b0 = p0 / tpb, b1 = (p1 - 1) / tpb;
    const int nblk = b1 - b0 - warp >= 0 ? (b1 - b0 - warp) / kAttnWarps + 1 : 0;

    if (lane == 0) {
        for (int s = 0; s < kMmaRing; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[warp][s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    // tensor-map rows: [block][layer][K|V][kv head][slot] rows of D halves
    const long long head_row = (a.layer_offset + (long long)h * tpb * D) / D;
    const long long block_rows = a.block_stride / D, kind_rows = a.kind_stride / D;
    // lane 0: start block i (physical id pb, read from the table beforehand)
    auto issue = [&](int i, int pb) {
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;
        }
        const int yk = int(pb * block_rows + head_row);
        const int yv = int(yk + kind_rows);
        const unsigned st = ring_s + unsigned((i % kMmaRing) * stage);
        const unsigned bar = s_u32(&bars[warp][i % kMmaRing]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(stage) : "memory");
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            tma_load_2d(st + b * box, &kv_map, b * 64, yk, bar);
            tma_load_2d(st + half_stage + b * box, &kv_map, b * 64, yv, bar);
        }
    };
    auto table = [&](int i) { return __ldg(a.tables + toff + b0 + warp + i * kAttnWarps); };
    if (lane == 0)
        for (int i = 0; i < kMmaRing && i < nblk; ++i) issue(i, table(i));

    const int gq = lane >> 2, tq = lane & 3;
    // Q^T as B fragments: lane holds head gq, d 16kk + 2tq + {0, 1} (+8);
    // scaled by 2^sh per head, hi + lo.
    unsigned qh[KS][2], ql[KS][2];
    float qinv0, qinv1;  // 2^-sh of heads 2tq and 2tq + 1 (this lane's S columns)
    {
        const bool row = gq < G;
        const float scale = rsqrtf(float(D));
        const float* qp = a.q + (long long)t * a.hq * D + (h * G + (row ? gq : 0)) * D;
        float v[KS][4];
        float mx = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                v[kk][e] = row ? qp[16 * kk + 2 * tq + e] * scale : 0.f;
                v[kk][2 + e] = row ? qp[16 * kk + 8 + 2 * tq + e] * scale : 0.f;
                mx = fmaxf(mx, fmaxf(fabsf(v[kk][e]), fabsf(v[kk][2 + e])));
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        int e2 = 0;
        if (mx > 0.f && isfinite(mx)) frexpf(mx, &e2);  // mx < 2^e2
        const int sh = max(-100, min(100, 15 - e2));
        const float up = exp2i(sh);
        const float inv = exp2i(-sh);
        qinv0 = __shfl_sync(0xffffffffu, inv, (2 * tq) * 4);
        qinv1 = __shfl_sync(0xffffffffu, inv, (2 * tq + 1) * 4);
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            split_f16x2(v[kk][0] * up, v[kk][1] * up, qh[kk][0], ql[kk][0]);
            split_f16x2(v[kk][2] * up, v[kk][3] * up, qh[kk][1], ql[kk][1]);
        }
    }

    float o[KS][4];  // O^T: d 16mt + gq (+8), heads 2tq, 2tq + 1
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2tq, 2tq + 1
    const int lr = lane & 7, lm = lane >> 3;  // ldmatrix: row within an 8x8 matrix, matrix index
    bool failed = false;
    for (int i = 0; i < nblk; ++i) {
        const int bi = b0 + warp + i * kAttnWarps;
        // the table entry of the block issued at the end of this iteration
        const int pnext = lane == 0 && i + kMmaRing < nblk ? table(i + kMmaRing) : 0;
        const unsigned parity = (i / kMmaRing) & 1;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[warp][i % kMmaRing], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const unsigned kst = ring_s + unsigned((i % kMmaRing) * stage);
        const unsigned vst = kst + half_stage;
        const int s_hi = min(tpb, p1 - bi * tpb);
        if (s_hi % 16) {
            // Slots past the visible end may hold anything (NaN included); P is
            // zero there, but 0 * NaN is NaN, so clear those V rows.
            unsigned char* vrows = ring + std::size_t(i % kMmaRing) * stage + half_stage;
            const int rows = ((s_hi + 15) & ~15) - s_hi;
            for (int idx = lane; idx < rows * NB * 8; idx += 32) {
                const int r = s_hi + idx / (NB * 8), c = idx % (NB * 8);
                *reinterpret_cast<uint4*>(vrows + (c >> 3) * box + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        for (int sub = 0; sub < s_hi; sub += 16) {
            // S^T: rows = positions sub + gq (+8), columns = heads 2tq, 2tq + 1
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                const int pos = sub + 8 * (lm & 1) + lr;
                const int c = 2 * kk + (lm >> 1);
                unsigned f[4];
                ldsm_x4(kst + (c >> 3) * box + pos * 128 + (((c & 7) ^ lr) << 4), f);
                mma16816(s, f, qh[kk][0], qh[kk][1]);
                mma16816(s, f, ql[kk][0], ql[kk][1]);
            }
            const bool va = sub + gq < s_hi, vb = sub + gq + 8 < s_hi;
            s[0] = va ? s[0] * qinv0 : -INFINITY;
            s[1] = va ? s[1] * qinv1 : -INFINITY;
            s[2] = vb ? s[2] * qinv0 : -INFINITY;
            s[3] = vb ? s[3] * qinv1 : -INFINITY;
            // Lazy reference (as attn_mma_i8_kernel): reduce and rescale only
            // when a score exceeds m by more than 4 ln 2; then P < 16.
            const bool over = s[0] > m0 + kLazyMargin || s[2] > m0 + kLazyMargin || s[1] > m1 + kLazyMargin ||
                              s[3] > m1 + kLazyMargin;
            if (__any_sync(0xffffffffu, over)) {
                float x0 = fmaxf(s[0], s[2]), x1 = fmaxf(s[1], s[3]);
#pragma unroll
                for (int o2 = 4; o2 < 32; o2 <<= 1) {
                    x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, o2));
                    x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o2));
                }
                const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
                const float al0 = m0 == -INFINITY ? 0.f : __expf(m0 - n0);
                const float al1 = m1 == -INFINITY ? 0.f : __expf(m1 - n1);
                m0 = n0;
                m1 = n1;
                l0 *= al0;
                l1 *= al1;
                float r0 = al0, r1 = al1;
                if constexpr (kPackLo) {  // lanes tq >= 2 hold the lo columns of heads 2tq - 4, 2tq - 3
                    const float u0 = __shfl_up_sync(0xffffffffu, r0, 2), u1 = __shfl_up_sync(0xffffffffu, r1, 2);
                    if (tq >= 2) {
                        r0 = u0;
                        r1 = u1;
                    }
                }
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    o[mt][0] *= r0;
                    o[mt][1] *= r1;
                    o[mt][2] *= r0;
                    o[mt][3] *= r1;
                }
            }
            const float pa0 = __expf(s[0] - m0), pa1 = __expf(s[1] - m1);
            const float pb0 = __expf(s[2] - m0), pb1 = __expf(s[3] - m1);
            l0 += pa0 + pb0;
            l1 += pa1 + pb1;
            // P^T (x 2^11 < 2^15) as the B operand: transpose the two 8x8 score tiles
            unsigned ha, la, hb, lb;
            split_f16x2(pa0 * 2048.f, pa1 * 2048.f, ha, la);
            split_f16x2(pb0 * 2048.f, pb1 * 2048.f, hb, lb);
            unsigned bh0, bh1, bl0 = 0, bl1 = 0;
            if constexpr (kPackLo) {
                const unsigned la2 = __shfl_up_sync(0xffffffffu, la, 2), lb2 = __shfl_up_sync(0xffffffffu, lb, 2);
                bh0 = movmatrix_t(tq < 2 ? ha : la2);
                bh1 = movmatrix_t(tq < 2 ? hb : lb2);
            } else {
                bh0 = movmatrix_t(ha);
                bh1 = movmatrix_t(hb);
                bl0 = movmatrix_t(la);
                bl1 = movmatrix_t(lb);
            }
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                // V^T tile [d 16mt.., positions sub..]: matrices (pos +0/+8) x (d +0/+8)
                const int pos = sub + 8 * (lm >> 1) + lr;
                const int c = 2 * mt + (lm & 1);
                unsigned f[4];
                ldsm_x4_t(vst + (c >> 3) * box + pos * 128 + (((c & 7) ^ lr) << 4), f);
                mma16816(o[mt], f, bh0, bh1);
                if constexpr (!kPackLo) mma16816(o[mt], f, bl0, bl1);
            }
        }
        __syncwarp();
        if (lane == 0 && i + kMmaRing < nblk) issue(i + kMmaRing, pnext);
    }
    if (lane == 0 && failed) {
        for (int i = 0; i < kMmaRing && i < nblk; ++i)
            for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[warp][i], 0) && !bar_try(&bars[warp][i], 1);
                 ++spin) {
            }
    }
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
    }
    __syncwarp();
    if constexpr (kPackLo) {  // hi columns (lanes tq < 2) plus the lo columns two lanes up
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[mt][e] += __shfl_down_sync(0xffffffffu, o[mt][e], 2);
    }
    // This warp's O (heads < G, scaled back by 2^-11) over its own first stage.
    float* acc = reinterpret_cast<float*>(ring);
    const int ha = 2 * tq, hb = 2 * tq + 1;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        if (ha < G) {
            acc[ha * D + 16 * mt + gq] = o[mt][0] * (1.f / 2048.f);
            acc[ha * D + 16 * mt + gq + 8] = o[mt][2] * (1.f / 2048.f);
        }
        if (hb < G) {
            acc[hb * D + 16 * mt + gq] = o[mt][1] * (1.f / 2048.f);
            acc[hb * D + 16 * mt + gq + 8] = o[mt][3] * (1.f / 2048.f);
        }
    }
    if (gq == 0) {
        s_m[warp][ha] = m0;
        s_l[warp][ha] = l0;
        s_m[warp][hb] = m1;
        s_l[warp][hb] = l1;
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
            const float f = __expf(s_m[w][g] - M);
            L = fmaf(s_l[w][g], f, L);
            A = fmaf(reinterpret_cast<const float*>(smem + std::size_t(w) * kMmaRing * stage)[g * D + e], f, A);
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

// Tensor-core attention for a chunk of consecutive query rows of one sequence
// (chunked prefill: row r of the chunk sees positions [0, v0 + r)), F16 KV,
// head_dim 64 or 128, blocks of a multiple of 16 slots, G = 1..8 query heads
// per KV head.
//
// CTA = 4 warps on one (chunk, KV head); each warp holds RW = floor(16 / G)
// rows x G query heads (16 query vectors when G divides 16; the spare
// vectors of G = 3, 5, 6, 7 repeat a live one and are not stored) on the M dimension of
// mma.m16n8k16 (the flash-attention layout: positions on N for S = Q K^T, on
// K for O += P V).  Every K/V tile is loaded once per CTA by TMA (boxes of 64
// halves x tpb slots, 128-byte swizzle, a ring of kChunkRing blocks filled by
// thread 0) and used by all four warps, so a chunk reads its KV once instead
// of once per row.  Q and P enter as exact hi + lo F16 pairs after
// power-of-two scaling (per query vector, P by 2^11), as in attn_mma_kernel;
// the softmax reference of a row moves only when a score exceeds it by more
// than 4 ln 2.
constexpr int kChunkRing = 4;

template <int D, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 2) attn_chunk_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                        AttnArgs a) {
    constexpr int NB = D / 64;   // 128-byte boxes per slot row
    constexpr int KS = D / 16;   // k-steps of S = Q K^T
    constexpr int NT = D / 8;    // n8 tiles of O
    constexpr int RW = 16 / G;   // rows per warp
    static_assert(D % 64 == 0 && G >= 1 && G <= 8, "chunk attention shape");
    extern __shared__ unsigned char att_raw[];
    __shared__ std::uint64_t bars[kChunkRing];
    const int tpb = a.tpb;
    const int box = tpb * 128;
    const int half_stage = NB * box;
    const int stage = 2 * half_stage;
    unsigned char* smem = att_raw + ((1024u - (s_u32(att_raw) & 1023u)) & 1023u);
    const unsigned ring_s = s_u32(smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, tq = lane & 3;
    const int lr = lane & 7, lm = lane >> 3;

    const int4 wk = a.chunk_work[blockIdx.x];
    const int t0 = wk.x, toff = wk.y, v0 = wk.z, nrows = wk.w;
    const int h = blockIdx.y;
    const int vlast = v0 + nrows - 1;              // positions the chunk's last row sees
    const int nblk = (vlast + tpb - 1) / tpb;
    const bool warp_live = warp * RW < nrows;      // warps without rows only help with the ring

    if (threadIdx.x == 0) {
        for (int s = 0; s < kChunkRing; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const long long head_row = (a.layer_offset + (long long)h * tpb * D) / D;
    const long long block_rows = a.block_stride / D, kind_rows = a.kind_stride / D;
    auto issue = [&](int i) {
        int pb = __ldg(a.tables + toff + i);
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;
        }
        const int yk = int(pb * block_rows + head_row);
        const int yv = int(yk + kind_rows);
        const unsigned st = ring_s + unsigned((i % kChunkRing) * stage);
        const unsigned bar = s_u32(&bars[i % kChunkRing]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(stage) : "memory");
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            tma_load_2d(st + b * box, &kv_map, b * 64, yk, bar);
            tma_load_2d(st + half_stage + b * box, &kv_map, b * 64, yv, bar);
        }
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < kChunkRing && i < nblk; ++i) issue(i);

    // This lane's query vectors: m = gq (row half 0) and gq + 8 (row half 1);
    // vector m is chunk row warp * RW + m / G, query head h * G + m % G.
    int vis[2];
    const float* qp[2];
    bool live[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int m = gq + 8 * hf;
        const bool vec = m < RW * G;  // a query vector of this warp (else a spare)
        const int r = warp * RW + (vec ? m / G : 0);
        live[hf] = vec && r < nrows;
        const int rr = live[hf] ? r : 0;  // spares and rows past the chunk compute row 0 and store nothing
        vis[hf] = v0 + rr;
        qp[hf] = a.q + (long long)(t0 + rr) * a.hq * D + (h * G + (vec ? m % G : 0)) * D;
    }
    // Q as A fragments (row-major 16 x 16 per k-step): a0 (gq, 2tq), a1 (gq + 8, 2tq),
    // a2 (gq, 2tq + 8), a3 (gq + 8, 2tq + 8); scaled per vector by 2^sh, hi + lo.
    unsigned qh[KS][4], ql[KS][4];
    float qinv[2];
    {
        const float scale = rsqrtf(float(D));
        float v[KS][8];
        float mx[2] = {0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const float2 x = *reinterpret_cast<const float2*>(qp[hf] + 16 * kk + 8 * c + 2 * tq);
                    v[kk][4 * c + 2 * hf] = x.x * scale;
                    v[kk][4 * c + 2 * hf + 1] = x.y * scale;
                    mx[hf] = fmaxf(mx[hf], fmaxf(fabsf(x.x * scale), fabsf(x.y * scale)));
                }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 1));
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 2));
        }
        float up[2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            int e2 = 0;
            if (mx[hf] > 0.f && isfinite(mx[hf])) frexpf(mx[hf], &e2);
            const int sh = max(-100, min(100, 15 - e2));
            up[hf] = exp2i(sh);
            qinv[hf] = exp2i(-sh);
        }
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            // v[kk]: [c][hf][2] -> fragments a0 (c0 hf0), a1 (c0 hf1), a2 (c1 hf0), a3 (c1 hf1)
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf)
                    split_f16x2(v[kk][4 * c + 2 * hf] * up[hf], v[kk][4 * c + 2 * hf + 1] * up[hf],
                                qh[kk][2 * c + hf], ql[kk][2 * c + hf]);
        }
    }

    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    bool failed = false;
    for (int i = 0; i < nblk; ++i) {
        const unsigned parity = (i / kChunkRing) & 1;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[i % kChunkRing], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const unsigned kst = ring_s + unsigned((i % kChunkRing) * stage);
        const unsigned vst = kst + half_stage;
        const int base = i * tpb;
        const int s_hi = min(tpb, vlast - base);
        if (s_hi % 16) {
            // V rows past the last row's visible end may hold anything (NaN
            // included): P is zero there, but 0 * NaN is NaN
            unsigned char* vrows = smem + std::size_t(i % kChunkRing) * stage + half_stage;
            const int rows = ((s_hi + 15) & ~15) - s_hi;
            for (int idx = threadIdx.x; idx < rows * NB * 8; idx += blockDim.x) {
                const int r = s_hi + idx / (NB * 8), c = idx % (NB * 8);
                *reinterpret_cast<uint4*>(vrows + (c >> 3) * box + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncthreads();
        }
        for (int sub = 0; warp_live && sub < s_hi; sub += 16) {
            float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                // K rows sub + 8 (lm >> 1) + lr, d chunk 2kk + (lm & 1): matrices
                // (pos 0-7, d 0-7), (pos 0-7, d 8-15), (pos 8-15, d 0-7), (pos 8-15, d 8-15)
                const int pos = sub + 8 * (lm >> 1) + lr;
                const int c = 2 * kk + (lm & 1);
                unsigned f[4];
                ldsm_x4(kst + (c >> 3) * box + pos * 128 + (((c & 7) ^ lr) << 4), f);
                mma16816(s[0], qh[kk], f[0], f[1]);
                mma16816(s[0], ql[kk], f[0], f[1]);
                mma16816(s[1], qh[kk], f[2], f[3]);
                mma16816(s[1], ql[kk], f[2], f[3]);
            }
            // scale back, mask: position p counts for vector (row) hf when p < vis[hf]
            bool over = false;
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hf = e >> 1;
                    const int p = base + sub + 8 * n + 2 * tq + (e & 1);
                    s[n][e] = p < vis[hf] ? s[n][e] * qinv[hf] : -INFINITY;
                    over |= s[n][e] > mrow[hf] + kLazyMargin;
                }
            if (__any_sync(0xffffffffu, over)) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float x = fmaxf(fmaxf(s[0][2 * hf], s[0][2 * hf + 1]), fmaxf(s[1][2 * hf], s[1][2 * hf + 1]));
                    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
                    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
                    const float nm = fmaxf(mrow[hf], x);
                    const float al = mrow[hf] == -INFINITY ? 0.f : __expf(mrow[hf] - nm);
                    mrow[hf] = nm;
                    lrow[hf] *= al;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        o[nt][2 * hf] *= al;
                        o[nt][2 * hf + 1] *= al;
                    }
                }
            }
            float p[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    p[n][e] = __expf(s[n][e] - mrow[e >> 1]);
                    lrow[e >> 1] += p[n][e];
                }
            // P (x 2^11 < 2^15) as A fragments: a0 (gq, pos 2tq) = p[0][0..1],
            // a1 (gq + 8) = p[0][2..3], a2 (gq, pos 2tq + 8) = p[1][0..1], a3 = p[1][2..3]
            unsigned ph[4], pl[4];
            split_f16x2(p[0][0] * 2048.f, p[0][1] * 2048.f, ph[0], pl[0]);
            split_f16x2(p[0][2] * 2048.f, p[0][3] * 2048.f, ph[1], pl[1]);
            split_f16x2(p[1][0] * 2048.f, p[1][1] * 2048.f, ph[2], pl[2]);
            split_f16x2(p[1][2] * 2048.f, p[1][3] * 2048.f, ph[3], pl[3]);
#pragma unroll
            for (int dt = 0; dt < NT / 2; ++dt) {
                // V^T fragments by transposed loads: matrices (pos 0-7, d 16dt..+7),
                // (pos 8-15, same d), (pos 0-7, d 16dt+8..), (pos 8-15, d 16dt+8..)
                const int pos = sub + 8 * (lm & 1) + lr;
                const int c = 2 * dt + (lm >> 1);
                unsigned f[4];
                ldsm_x4_t(vst + (c >> 3) * box + pos * 128 + (((c & 7) ^ lr) << 4), f);
                mma16816(o[2 * dt], ph, f[0], f[1]);
                mma16816(o[2 * dt], pl, f[0], f[1]);
                mma16816(o[2 * dt + 1], ph, f[2], f[3]);
                mma16816(o[2 * dt + 1], pl, f[2], f[3]);
            }
        }
        __syncthreads();  // every warp is done with this stage
        if (threadIdx.x == 0 && i + kChunkRing < nblk) issue(i + kChunkRing);
    }
    if (failed) {
        // wait (bounded) for this CTA's copies still in flight before exiting
        if (threadIdx.x == 0)
            for (int i = 0; i < kChunkRing && i < nblk; ++i)
                for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[i], 0) && !bar_try(&bars[i], 1); ++spin) {
                }
        return;
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        lrow[hf] += __shfl_xor_sync(0xffffffffu, lrow[hf], 1);
        lrow[hf] += __shfl_xor_sync(0xffffffffu, lrow[hf], 2);
    }
    if (!warp_live) return;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        if (!live[hf]) continue;
        const int m = gq + 8 * hf;
        const int r = warp * RW + m / G;  // live: m < RW * G
        const float inv = 1.f / (lrow[hf] * 2048.f);
        float* op = a.out + (long long)(t0 + r) * a.hq * D + (h * G + m % G) * D;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float2*>(op + 8 * nt + 2 * tq) = make_float2(o[nt][2 * hf] * inv, o[nt][2 * hf + 1] * inv);
    }
}

// The chunk kernel for F32 pools (the reference's KV format).  Same CTA,
// work items and softmax as attn_chunk_kernel; the K/V tiles are F32 rows in
// shared memory (TMA boxes of 32 floats x tpb slots, 128-byte swizzle), and
// the MMA operands are built from them in registers as exact hi + lo F16
// pairs after a per-tile power-of-two scaling: S = Q_hi K_hi + Q_lo K_hi +
// Q_hi K_lo and O += P_hi V_hi + P_lo V_hi + P_hi V_lo (the lo x lo products
// are below 2^-22 of the result), so K and V keep about 22 of their 24 bits.
// The tile's scale of K (or V) is the power of two that brings its largest
// |value| below 2^15, found by one pass over the tile in shared memory.
template <int D, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 2) attn_chunk_f32_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                            AttnArgs a) {
    constexpr int NB = D / 32;   // 128-byte boxes (32 floats) per slot row
    constexpr int KS = D / 16;   // k-steps of S = Q K^T
    constexpr int NT = D / 8;    // n8 tiles of O
    constexpr int RW = 16 / G;   // rows per warp
    static_assert(D % 32 == 0 && G >= 1 && G <= 8, "chunk attention shape");
    extern __shared__ unsigned char att_raw[];
    __shared__ std::uint64_t bars[kChunkRing];
    __shared__ float tile_scale[2];  // 2^-e of the current tile's K and V maxima
    const int tpb = a.tpb;
    const int box = tpb * 128;
    const int half_stage = NB * box;
    const int stage = 2 * half_stage;
    unsigned char* smem = att_raw + ((1024u - (s_u32(att_raw) & 1023u)) & 1023u);
    const unsigned ring_s = s_u32(smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, tq = lane & 3;

    const int4 wk = a.chunk_work[blockIdx.x];
    const int t0 = wk.x, toff = wk.y, v0 = wk.z, nrows = wk.w;
    const int h = blockIdx.y;
    const int vlast = v0 + nrows - 1;
    const int nblk = (vlast + tpb - 1) / tpb;
    const bool warp_live = warp * RW < nrows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kChunkRing; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const long long head_row = (a.layer_offset + (long long)h * tpb * D) / D;
    const long long block_rows = a.block_stride / D, kind_rows = a.kind_stride / D;
    auto issue = [&](int i) {
        int pb = __ldg(a.tables + toff + i);
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;
        }
        const int yk = int(pb * block_rows + head_row);
        const int yv = int(yk + kind_rows);
        const unsigned st = ring_s + unsigned((i % kChunkRing) * stage);
        const unsigned bar = s_u32(&bars[i % kChunkRing]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(stage) : "memory");
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            tma_load_2d(st + b * box, &kv_map, b * 32, yk, bar);
            tma_load_2d(st + half_stage + b * box, &kv_map, b * 32, yv, bar);
        }
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < kChunkRing && i < nblk; ++i) issue(i);

    int vis[2];
    const float* qp[2];
    bool live[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int m = gq + 8 * hf;
        const bool vec = m < RW * G;
        const int r = warp * RW + (vec ? m / G : 0);
        live[hf] = vec && r < nrows;
        const int rr = live[hf] ? r : 0;
        vis[hf] = v0 + rr;
        qp[hf] = a.q + (long long)(t0 + rr) * a.hq * D + (h * G + (vec ? m % G : 0)) * D;
    }
    unsigned qh[KS][4], ql[KS][4];
    float qinv[2];
    {
        const float scale = rsqrtf(float(D));
        float v[KS][8];
        float mx[2] = {0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const float2 x = *reinterpret_cast<const float2*>(qp[hf] + 16 * kk + 8 * c + 2 * tq);
                    v[kk][4 * c + 2 * hf] = x.x * scale;
                    v[kk][4 * c + 2 * hf + 1] = x.y * scale;
                    mx[hf] = fmaxf(mx[hf], fmaxf(fabsf(x.x * scale), fabsf(x.y * scale)));
                }
        float up[2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 1));
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 2));
            int e2 = 0;
            if (mx[hf] > 0.f && isfinite(mx[hf])) frexpf(mx[hf], &e2);
            const int sh = max(-100, min(100, 15 - e2));
            up[hf] = exp2i(sh);
            qinv[hf] = exp2i(-sh);
        }
#pragma unroll
        for (int kk = 0; kk < KS; ++kk)
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf)
                    split_f16x2(v[kk][4 * c + 2 * hf] * up[hf], v[kk][4 * c + 2 * hf + 1] * up[hf], qh[kk][2 * c + hf],
                                ql[kk][2 * c + hf]);
    }
    // element (pos, d) of a K or V tile: box d / 32, 16-byte chunk (d % 32) / 4 swizzled with the row
    auto f32_at = [&](const unsigned char* tile, int pos, int d) -> const float* {
        return reinterpret_cast<const float*>(tile + (d >> 5) * box + pos * 128 + ((((d & 31) >> 2) ^ (pos & 7)) << 4) +
                                              (d & 3) * 4);
    };

    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    bool failed = false;
    for (int i = 0; i < nblk; ++i) {
        const unsigned parity = (i / kChunkRing) & 1;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[i % kChunkRing], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const unsigned char* kst = smem + std::size_t(i % kChunkRing) * stage;
        const unsigned char* vst = kst + half_stage;
        const int base = i * tpb;
        const int s_hi = min(tpb, vlast - base);
        {
            // rows past the last row's visible end may hold anything: zero them
            // (K and V) so that the tile maxima and 0 * V stay finite; then the
            // power-of-two scales of this tile's K and V
            unsigned char* krows = smem + std::size_t(i % kChunkRing) * stage;
            const int pad = ((s_hi + 15) & ~15) - s_hi;
            for (int idx = threadIdx.x; idx < 2 * pad * NB * 8; idx += blockDim.x) {
                const int kind = idx / (pad * NB * 8), rem = idx % (pad * NB * 8);
                const int r = s_hi + rem / (NB * 8), c = rem % (NB * 8);
                *reinterpret_cast<uint4*>(krows + kind * half_stage + (c >> 3) * box + r * 128 + (c & 7) * 16) =
                    make_uint4(0, 0, 0, 0);
            }
            float mk = 0.f, mv = 0.f;
            for (int idx = threadIdx.x; idx < s_hi * D / 4; idx += blockDim.x) {
                const int r = idx / (D / 4), c = idx % (D / 4);  // 16-byte chunk c of row r (any order will do)
                const float4 kq = *reinterpret_cast<const float4*>(krows + (c >> 3) * box + r * 128 + (c & 7) * 16);
                const float4 vq = *reinterpret_cast<const float4*>(krows + half_stage + (c >> 3) * box + r * 128 + (c & 7) * 16);
                mk = fmaxf(mk, fmaxf(fmaxf(fabsf(kq.x), fabsf(kq.y)), fmaxf(fabsf(kq.z), fabsf(kq.w))));
                mv = fmaxf(mv, fmaxf(fmaxf(fabsf(vq.x), fabsf(vq.y)), fmaxf(fabsf(vq.z), fabsf(vq.w))));
            }
            for (int o2 = 16; o2; o2 >>= 1) {
                mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o2));
                mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o2));
            }
            __shared__ float red[2][kAttnWarps];
            if (lane == 0) {
                red[0][warp] = mk;
                red[1][warp] = mv;
            }
            __syncthreads();
            if (threadIdx.x < 2) {
                float m = 0.f;
                for (int w = 0; w < kAttnWarps; ++w) m = fmaxf(m, red[threadIdx.x][w]);
                int e2 = 0;
                if (m > 0.f && isfinite(m)) frexpf(m, &e2);
                tile_scale[threadIdx.x] = exp2i(max(-100, min(100, 15 - e2)));
            }
            __syncthreads();
        }
        const float ks_up = tile_scale[0], vs_up = tile_scale[1];
        const float ks_inv = 1.f / ks_up, vs_inv = 1.f / vs_up;  // exact: powers of two
        for (int sub = 0; warp_live && sub < s_hi; sub += 16) {
            float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    // B = K^T: (k = d 16kk + 2tq, + 1 | + 8, + 9; n = position sub + 8n + gq)
                    const int pos = sub + 8 * n + gq;
                    const float2 k0 = *reinterpret_cast<const float2*>(f32_at(kst, pos, 16 * kk + 2 * tq));
                    const float2 k1 = *reinterpret_cast<const float2*>(f32_at(kst, pos, 16 * kk + 8 + 2 * tq));
                    unsigned bh0, bl0, bh1, bl1;
                    split_f16x2(k0.x * ks_up, k0.y * ks_up, bh0, bl0);
                    split_f16x2(k1.x * ks_up, k1.y * ks_up, bh1, bl1);
                    mma16816(s[n], qh[kk], bh0, bh1);
                    mma16816(s[n], ql[kk], bh0, bh1);
                    mma16816(s[n], qh[kk], bl0, bl1);
                }
            }
            bool over = false;
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hf = e >> 1;
                    const int p = base + sub + 8 * n + 2 * tq + (e & 1);
                    s[n][e] = p < vis[hf] ? s[n][e] * qinv[hf] * ks_inv : -INFINITY;
                    over |= s[n][e] > mrow[hf] + kLazyMargin;
                }
            if (__any_sync(0xffffffffu, over)) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float x = fmaxf(fmaxf(s[0][2 * hf], s[0][2 * hf + 1]), fmaxf(s[1][2 * hf], s[1][2 * hf + 1]));
                    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
                    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
                    const float nm = fmaxf(mrow[hf], x);
                    const float al = mrow[hf] == -INFINITY ? 0.f : __expf(mrow[hf] - nm);
                    mrow[hf] = nm;
                    lrow[hf] *= al;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        o[nt][2 * hf] *= al;
                        o[nt][2 * hf + 1] *= al;
                    }
                }
            }
            float p[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    p[n][e] = __expf(s[n][e] - mrow[e >> 1]);
                    lrow[e >> 1] += p[n][e];
                }
            unsigned ph[4], pl[4];
            split_f16x2(p[0][0] * 2048.f, p[0][1] * 2048.f, ph[0], pl[0]);
            split_f16x2(p[0][2] * 2048.f, p[0][3] * 2048.f, ph[1], pl[1]);
            split_f16x2(p[1][0] * 2048.f, p[1][1] * 2048.f, ph[2], pl[2]);
            split_f16x2(p[1][2] * 2048.f, p[1][3] * 2048.f, ph[3], pl[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                // B = V: (k = position sub + 2tq, + 1 | + 8, + 9; n = d 8nt + gq), scaled by the tile's power of two
                const int d = 8 * nt + gq;
                const float va = *f32_at(vst, sub + 2 * tq, d);
                const float vb = *f32_at(vst, sub + 2 * tq + 1, d);
                const float vc = *f32_at(vst, sub + 2 * tq + 8, d);
                const float vd = *f32_at(vst, sub + 2 * tq + 9, d);
                unsigned bh0, bl0, bh1, bl1;
                split_f16x2(va * vs_up, vb * vs_up, bh0, bl0);
                split_f16x2(vc * vs_up, vd * vs_up, bh1, bl1);
                float t4[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(t4, ph, bh0, bh1);
                mma16816(t4, pl, bh0, bh1);
                mma16816(t4, ph, bl0, bl1);
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nt][e] = fmaf(t4[e], vs_inv, o[nt][e]);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && i + kChunkRing < nblk) issue(i + kChunkRing);
    }
    if (failed) {
        if (threadIdx.x == 0)
            for (int i = 0; i < kChunkRing && i < nblk; ++i)
                for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[i], 0) && !bar_try(&bars[i], 1); ++spin) {
                }
        return;
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        lrow[hf] += __shfl_xor_sync(0xffffffffu, lrow[hf], 1);
        lrow[hf] += __shfl_xor_sync(0xffffffffu, lrow[hf], 2);
    }
    if (!warp_live) return;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        if (!live[hf]) continue;
        const int m = gq + 8 * hf;
        const int r = warp * RW + m / G;
        const float inv = 1.f / (lrow[hf] * 2048.f);
        float* op = a.out + (long long)(t0 + r) * a.hq * D + (h * G + m % G) * D;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float2*>(op + 8 * nt + 2 * tq) = make_float2(o[nt][2 * hf] * inv, o[nt][2 * hf + 1] * inv);
    }
}

// Tensor-core paged attention for int8 KV (head_dim 64 or 128, blocks of a
// multiple of 16 slots).  CTA and ring as attn_mma_kernel (three stages
// per warp, four CTAs per SM: a stage is half the bytes); one TMA box per K or V run of a block (rows of
// D bytes, 128- or 64-byte swizzle) plus a bulk copy of the block's 2 x tpb
// row scales.  The scales enter outside the MMAs:
//   S^T = scale_k[pos] * (code_K . Q^T) on the integer tensor path
// (mma.m16n8k32, s8 x u8/s8 -> s32): the K codes are the A operand straight
// from ldmatrix, Q^T is 22-bit fixed point (per head 2^sh) as three byte
// digits (low two unsigned, top signed), so each product is exact and the
// three digit sums combine in F32;
//   O^T += code_V^T . P'^T on the F16 path (codes in [-127, 127] are exact
// F16): ldmatrix.trans of the int8 rows gives each lane two positions x two
// d per word, widened to F16 pairs by a byte permute (0x64XX = 1024 + XX)
// and one subtraction; the m rows of a tile are d = 2g (row g) and 2g + 1
// (row g + 8).  P' = P * scale_v * 2^(11 - ev) with ev a running
// power-of-two bound of the V scales seen, so P' < 2^15 splits into exact
// hi + lo F16 as P does for F16 KV.
//   The softmax reference m (per head) and ev are lazy: a tile reduces and
// rescales only when one of its scores exceeds m by more than 4 ln 2 (then
// m becomes the maximum so far) or one of its V scales reaches 2^ev; other
// tiles use P = e^(s - m) < 16 as they are.  Any reference gives the same
// softmax, since O and the running sum share it.
constexpr int kI8Ring = 3;

// Shared-memory byte offset of (row, byte) in a tile of rows of RB bytes
// written by TMA with the RB-byte swizzle (RB = 128 or 64).
template <int RB>
__device__ __forceinline__ unsigned swz_off(int row, int byte) {
    if constexpr (RB == 128) return unsigned(row * 128 + ((((byte >> 4) ^ row) & 7) << 4) + (byte & 15));
    else return unsigned(row * 64 + ((((byte >> 4) ^ (row >> 1)) & 3) << 4) + (byte & 15));
}
// F16 pair from bytes of a biased word (code + 128 per byte) picked by
// `sel` next to 0x64 bytes: 0x64XX is 1024 + XX, exact; minus 1152.
__device__ __forceinline__ unsigned i8pair_f16(unsigned biased, unsigned sel) {
    const unsigned w = __byte_perm(biased, 0x64646464u, sel);
    __half2 h = *reinterpret_cast<const __half2*>(&w);
    h = __hsub2(h, __half2half2(__ushort_as_half(0x6480)));  // 1152
    return *reinterpret_cast<const unsigned*>(&h);
}
// d += A b for one m16n8k32 integer tile (A s8 row-major 16x32, b col-major
// 32x8, u8 or s8).
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int D, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 4) attn_mma_i8_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                         AttnArgs a) {
    constexpr int KS = D / 16;
    // G <= 4: columns 4..7 of P'^T carry the lo parts of heads 0..3, so one
    // MMA per V tile takes hi and lo (O^T columns 4..7 are added back at the end)
    constexpr bool kPackLo = G <= 4;
    static_assert((D == 64 || D == 128) && G >= 1 && G <= 8, "int8 tensor-core attention shape");
    extern __shared__ unsigned char att_raw[];
    __shared__ std::uint64_t bars[kAttnWarps][kI8Ring];
    __shared__ float s_m[kAttnWarps][8], s_l[kAttnWarps][8];
    const int tpb = a.tpb;
    const int run = tpb * D;           // bytes of one K (or V) run of a block
    const int stage = 2 * run;
    unsigned char* smem = att_raw + ((1024u - (s_u32(att_raw) & 1023u)) & 1023u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned char* ring = smem + std::size_t(warp) * kI8Ring * stage;
    const unsigned ring_s = s_u32(ring);
    // scales: [warp][stage][K | V][tpb] floats after all rings
    float* scl = reinterpret_cast<float*>(smem + std::size_t(kAttnWarps) * kI8Ring * stage) +
                 std::size_t(warp) * kI8Ring * 2 * tpb;

    const int4 wk = a.work[blockIdx.x];
    const int part = a.work_part[blockIdx.x];
    const int t = wk.x, toff = wk.y, p0 = wk.z, p1 = wk.w;
    const int h = blockIdx.y;
    const int b0 = p0 / tpb, b1 = (p1 - 1) / tpb;
    const int nblk = b1 - b0 - warp >= 0 ? (b1 - b0 - warp) / kAttnWarps + 1 : 0;

    if (lane == 0) {
        for (int s = 0; s < kI8Ring; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&bars[warp][s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    const long long head_row = (a.layer_offset + (long long)h * tpb * D) / D;
    const long long block_rows = a.block_stride / D, kind_rows = a.kind_stride / D;
    // lane 0: start a block (physical id pb, read from the table beforehand) into stage st
    auto issue = [&](int st, int pb) {
        if (pb < 0 || pb >= a.max_blocks) {
            atomicExch(a.err, 2);
            pb = 0;
        }
        const long long yk = pb * block_rows + head_row;
        const long long yv = yk + kind_rows;
        const unsigned dst = ring_s + unsigned(st * stage);
        std::uint64_t* bar = &bars[warp][st];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(bar)),
                     "r"(stage + 8 * tpb)
                     : "memory");
        tma_load_2d(dst, &kv_map, 0, int(yk), s_u32(bar));
        tma_load_2d(dst + run, &kv_map, 0, int(yv), s_u32(bar));
        bulk_g2s(scl + st * 2 * tpb, a.kv_scales + yk, unsigned(4 * tpb), bar);
        bulk_g2s(scl + st * 2 * tpb + tpb, a.kv_scales + yv, unsigned(4 * tpb), bar);
    };
    auto table = [&](int i) { return __ldg(a.tables + toff + b0 + warp + i * kAttnWarps); };
    if (lane == 0)
        for (int i = 0; i < kI8Ring && i < nblk; ++i) issue(i, table(i));  // block i into stage i

    const int gq = lane >> 2, tq = lane & 3;
    // Q^T in three byte digits (B fragments of m16n8k32): step kk, lane
    // (gq, tq) holds head gq, d 32kk + 4tq + {0..3} (reg 0) and 32kk + 16 +
    // 4tq + {0..3} (reg 1) of x = rint(q / sqrt(D) * 2^sh), |x| <= 2^21 per
    // head; digit j is byte j of x (0, 1 unsigned; 2 signed, two's complement).
    constexpr int K32 = D / 32;
    unsigned qd[K32][3][2];
    float qinv0, qinv1;  // 2^-sh of heads 2tq and 2tq + 1 (this lane's S columns)
    {
        const bool row = gq < G;
        const float scale = rsqrtf(float(D));
        const float* qp = a.q + (long long)t * a.hq * D + (h * G + (row ? gq : 0)) * D;
        float v[K32][2][4];
        float mx = 0.f;
#pragma unroll
        for (int kk = 0; kk < K32; ++kk)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const float4 f = row ? *reinterpret_cast<const float4*>(qp + 32 * kk + 16 * r + 4 * tq)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                v[kk][r][0] = f.x * scale;
                v[kk][r][1] = f.y * scale;
                v[kk][r][2] = f.z * scale;
                v[kk][r][3] = f.w * scale;
#pragma unroll
                for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fabsf(v[kk][r][e]));
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        int e2 = 0;
        if (mx > 0.f && isfinite(mx)) frexpf(mx, &e2);  // mx < 2^e2
        const int sh = max(-100, min(100, 21 - e2));
        const float up = exp2i(sh);
        const float inv = exp2i(-sh);
        qinv0 = __shfl_sync(0xffffffffu, inv, (2 * tq) * 4);
        qinv1 = __shfl_sync(0xffffffffu, inv, (2 * tq + 1) * 4);
#pragma unroll
        for (int kk = 0; kk < K32; ++kk)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                int x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) x[e] = __float2int_rn(v[kk][r][e] * up);
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    unsigned w = 0;
#pragma unroll
                    for (int e = 0; e < 4; ++e) w |= ((unsigned(x[e]) >> (8 * j)) & 255u) << (8 * e);
                    qd[kk][j][r] = w;
                }
            }
    }

    float o[KS][4];  // O^T tile mt: d 16mt + 2gq (regs 0, 1), + 1 (regs 2, 3); heads 2tq, 2tq + 1
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    int ev = -1000;     // running exponent bound of the V scales (none yet)
    float vlim = 0.f;   // 2^ev
    float up = 0.f;     // 2^(11 - ev)
    const int lr = lane & 7, lm = lane >> 3;  // ldmatrix: row within an 8x8 matrix, matrix index
    // This lane's ldmatrix row address within a 16-row tile, per 32 columns;
    // the swizzle depends on the row's low four bits only, so a tile at row
    // `sub` (a multiple of 16) adds sub * D.
    unsigned ofs[K32];
#pragma unroll
    for (int kk = 0; kk < K32; ++kk) ofs[kk] = swz_off<D>(8 * (lm & 1) + lr, 32 * kk + 16 * (lm >> 1));
    bool failed = false;
    int st = 0;           // stage of block i
    unsigned parity = 0;  // its mbarrier phase
    for (int i = 0; i < nblk; ++i) {
        const int bi = b0 + warp + i * kAttnWarps;
        // the table entry of the block issued at the end of this iteration,
        // loaded now so its latency hides behind the compute
        const int pnext = lane == 0 && i + kI8Ring < nblk ? table(i + kI8Ring) : 0;
        unsigned ok = 0;
        for (unsigned spin = 0; spin < kAttnSpin; ++spin) {
            if (bar_try(&bars[warp][st], parity)) {
                ok = 1;
                break;
            }
            if (spin > 32) __nanosleep(32);
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicExch(a.err, 4);
            failed = true;
            break;
        }
        const unsigned kst = ring_s + unsigned(st * stage);
        const unsigned vst = kst + run;
        const float* sk = scl + st * 2 * tpb;
        const float* sv = sk + tpb;
        const int s_hi = min(tpb, p1 - bi * tpb);
        for (int sub = 0; sub < s_hi; sub += 16) {
            const int pa = sub + gq, pb = sub + gq + 8;
            const bool va = pa < s_hi, vb = pb < s_hi;
            // S^T: rows = positions sub + gq (+8), columns = heads 2tq, 2tq + 1
            int ai[3][4] = {};
#pragma unroll
            for (int kk = 0; kk < K32; ++kk) {
                unsigned f[4];
                ldsm_x4(kst + unsigned(sub * D) + ofs[kk], f);
                mma_s8u8(ai[0], f, qd[kk][0][0], qd[kk][0][1]);
                mma_s8u8(ai[1], f, qd[kk][1][0], qd[kk][1][1]);
                mma_s8s8(ai[2], f, qd[kk][2][0], qd[kk][2][1]);
            }
            float s[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                s[e] = fmaf(float(ai[2][e]), 65536.f, fmaf(float(ai[1][e]), 256.f, float(ai[0][e])));
            const float ka = sk[pa], kb = sk[pb];
            s[0] = va ? s[0] * qinv0 * ka : -INFINITY;
            s[1] = va ? s[1] * qinv1 * ka : -INFINITY;
            s[2] = vb ? s[2] * qinv0 * kb : -INFINITY;
            s[3] = vb ? s[3] * qinv1 * kb : -INFINITY;
            const float fa = va ? sv[pa] : 0.f, fb = vb ? sv[pb] : 0.f;
            // The reference points m0, m1 (heads 2tq, 2tq + 1) and 2^ev move
            // only when a score exceeds its reference by more than 4 ln 2 or a
            // V scale reaches 2^ev: most tiles take no reduction and no rescale.
            // Afterwards P = e^(s - m) < 16 and P' = P * scale_v * 2^(11 - ev) < 2^15.
            const bool over = s[0] > m0 + kLazyMargin || s[2] > m0 + kLazyMargin || s[1] > m1 + kLazyMargin ||
                              s[3] > m1 + kLazyMargin || fmaxf(fa, fb) >= vlim;
            if (__any_sync(0xffffffffu, over)) {
                float x0 = fmaxf(s[0], s[2]), x1 = fmaxf(s[1], s[3]);
                float vm = fmaxf(fa, fb);
#pragma unroll
                for (int o2 = 4; o2 < 32; o2 <<= 1) {
                    x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, o2));
                    x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o2));
                    vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, o2));
                }
                // vm < 2^et from the exponent field (subnormals and 0 give -126,
                // clamped to -100 like every bound below 2^-100)
                const int et = max(-100, min(126, int((__float_as_uint(vm) >> 23) & 255u) - 126));
                float grow = 1.f;
                if (et > ev) {
                    grow = ev - et >= -126 ? exp2i(ev - et) : 0.f;
                    ev = et;
                    vlim = exp2i(ev);
                    up = exp2i(11 - ev);
                }
                const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
                const float al0 = m0 == -INFINITY ? 0.f : __expf(m0 - n0);
                const float al1 = m1 == -INFINITY ? 0.f : __expf(m1 - n1);
                m0 = n0;
                m1 = n1;
                l0 *= al0;
                l1 *= al1;
                float r0 = al0 * grow, r1 = al1 * grow;
                if constexpr (kPackLo) {  // lanes tq >= 2 hold the lo columns of heads 2tq - 4, 2tq - 3
                    const float u0 = __shfl_up_sync(0xffffffffu, r0, 2), u1 = __shfl_up_sync(0xffffffffu, r1, 2);
                    if (tq >= 2) {
                        r0 = u0;
                        r1 = u1;
                    }
                }
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    o[mt][0] *= r0;
                    o[mt][1] *= r1;
                    o[mt][2] *= r0;
                    o[mt][3] *= r1;
                }
            }
            const float pa0 = __expf(s[0] - m0), pa1 = __expf(s[1] - m1);
            const float pb0 = __expf(s[2] - m0), pb1 = __expf(s[3] - m1);
            l0 += pa0 + pb0;
            l1 += pa1 + pb1;
            // positions past the end have P = 0 and scale 0
            const float wa = fa * up, wb = fb * up;
            unsigned ha, la, hb, lb;
            split_f16x2(pa0 * wa, pa1 * wa, ha, la);
            split_f16x2(pb0 * wb, pb1 * wb, hb, lb);
            unsigned bh0, bh1, bl0 = 0, bl1 = 0;
            if constexpr (kPackLo) {
                const unsigned la2 = __shfl_up_sync(0xffffffffu, la, 2), lb2 = __shfl_up_sync(0xffffffffu, lb, 2);
                bh0 = movmatrix_t(tq < 2 ? ha : la2);
                bh1 = movmatrix_t(tq < 2 ? hb : lb2);
            } else {
                bh0 = movmatrix_t(ha);
                bh1 = movmatrix_t(hb);
                bl0 = movmatrix_t(la);
                bl1 = movmatrix_t(lb);
            }
#pragma unroll
            for (int j = 0; j < D / 32; ++j) {
                // matrices 0, 1: positions sub + 0..7, 8..15 of d 32j..32j+15; 2, 3: of d 32j+16..
                unsigned w[4];
                ldsm_x4_t(vst + unsigned(sub * D) + ofs[j], w);
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    // word: (pos 2tq, d 2gq), (2tq, 2gq+1), (2tq+1, 2gq), (2tq+1, 2gq+1)
                    const unsigned u0 = w[2 * hf] ^ 0x80808080u, u1 = w[2 * hf + 1] ^ 0x80808080u;
                    const unsigned f[4] = {i8pair_f16(u0, 0x4240), i8pair_f16(u0, 0x4341), i8pair_f16(u1, 0x4240),
                                           i8pair_f16(u1, 0x4341)};
                    mma16816(o[2 * j + hf], f, bh0, bh1);
                    if constexpr (!kPackLo) mma16816(o[2 * j + hf], f, bl0, bl1);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + kI8Ring < nblk) issue(st, pnext);
        if (++st == kI8Ring) {
            st = 0;
            parity ^= 1;
        }
    }
    if (lane == 0 && failed) {
        for (int i = 0; i < kI8Ring && i < nblk; ++i)
            for (unsigned spin = 0; spin < kAttnSpin && !bar_try(&bars[warp][i], 0) && !bar_try(&bars[warp][i], 1);
                 ++spin) {
            }
    }
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
    }
    __syncwarp();
    if constexpr (kPackLo) {  // hi columns (lanes tq < 2) plus the lo columns two lanes up
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[mt][e] += __shfl_down_sync(0xffffffffu, o[mt][e], 2);
    }
    // This warp's O (heads < G, scaled back by 2^(ev - 11)) over its own ring.
    float* acc = reinterpret_cast<float*>(ring);
    const float down = ev == -1000 ? 0.f : exp2i(ev - 11);
    const int ha = 2 * tq, hb = 2 * tq + 1;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        const int d = 16 * mt + 2 * gq;
        if (ha < G) {
            acc[ha * D + d] = o[mt][0] * down;
            acc[ha * D + d + 1] = o[mt][2] * down;
        }
        if (hb < G) {
            acc[hb * D + d] = o[mt][1] * down;
            acc[hb * D + d + 1] = o[mt][3] * down;
        }
    }
    if (gq == 0) {
        s_m[warp][ha] = m0;
        s_l[warp][ha] = l0;
        s_m[warp][hb] = m1;
        s_l[warp][hb] = l1;
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
            const float f = __expf(s_m[w][g] - M);
            L = fmaf(s_l[w][g], f, L);
            A = fmaf(reinterpret_cast<const float*>(smem + std::size_t(w) * kI8Ring * stage)[g * D + e], f, A);
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

// The dynamic shared-memory limit is a per-device function attribute: set it
// on every launch (a host-side call of about a microsecond).
template <int D, typename KV, int G>
void run_pipe(const AttnArgs& a, dim3 grid, int smem, cudaStream_t s) {
    TVARA_CUDA(cudaFuncSetAttribute(attn_pipe_kernel<D, KV, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attn_pipe_kernel<D, KV, G><<<grid, kAttnWarps * 32, smem, s>>>(a);
}

template <int D, typename KV, int G>
void run_xpose(const AttnArgs& a, dim3 grid, int smem, cudaStream_t s) {
    TVARA_CUDA(cudaFuncSetAttribute(attn_xpose_kernel<D, KV, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attn_xpose_kernel<D, KV, G><<<grid, kAttnWarps * 32, smem, s>>>(a);
}

// The F16 pool as a 2-D tensor of rows of D halves (one row = one slot of one
// KV head of one layer of one block), read in boxes of 64 halves x tpb rows
// with the 128-byte swizzle.
CUtensorMap kv_map_f16(const AttnArgs& a, int D) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(D), cuuint64_t((long long)a.max_blocks * (a.block_stride / D))};
    const cuuint64_t strides[1] = {cuuint64_t(D) * 2};
    const cuuint32_t box[2] = {64, cuuint32_t(a.tpb)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.kv), dims,
                                            strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

constexpr long long mma_smem_bytes(int D, int tpb) {
    return 1024 + (long long)kAttnWarps * kMmaRing * 2 * (D / 64) * tpb * 128;
}

// Whether the tensor-core kernel takes these arguments: F16 pool, head_dim 64
// or 128, blocks of a multiple of 16 slots, rows addressable by the map.
bool mma_ok(const AttnArgs& a) {
    if (!a.kv_f16 || (a.dim != 64 && a.dim != 128) || a.tpb % 16 || a.tpb > 256) return false;
    if (reinterpret_cast<std::uintptr_t>(a.kv) % 16 || mma_smem_bytes(a.dim, a.tpb) > 200 * 1024) return false;
    return (long long)a.max_blocks * (a.block_stride / a.dim) < (1ll << 31);
}

template <int D, int G>
void run_mma(const AttnArgs& a, dim3 grid, cudaStream_t s) {
    const int smem = int(mma_smem_bytes(D, a.tpb));
    TVARA_CUDA(cudaFuncSetAttribute(attn_mma_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const CUtensorMap map = kv_map_f16(a, D);
    attn_mma_kernel<D, G><<<grid, kAttnWarps * 32, smem, s>>>(map, a);
}

// The int8 pool as rows of D bytes, one box per K or V run of a block (tpb
// rows), swizzled over the row width (128 or 64 bytes).
CUtensorMap kv_map_i8(const AttnArgs& a, int D) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(D), cuuint64_t((long long)a.max_blocks * (a.block_stride / D))};
    const cuuint64_t strides[1] = {cuuint64_t(D)};
    const cuuint32_t box[2] = {cuuint32_t(D), cuuint32_t(a.tpb)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a.kv), dims,
                                            strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

constexpr long long mma_i8_smem_bytes(int D, int tpb) {
    return 1024 + (long long)kAttnWarps * kI8Ring * (2 * tpb * D + 8 * tpb);
}

// Whether the int8 tensor-core kernel takes these arguments: head_dim 64 or
// 128, blocks of a multiple of 16 slots, 16-byte aligned pool, scales and
// queries, and every scale run of a block 16-byte aligned (row offsets of
// blocks, layers and kinds multiples of 4 rows).
bool mma_i8_ok(const AttnArgs& a) {
    if (!a.kv_i8 || (a.dim != 64 && a.dim != 128) || a.tpb % 16 || a.tpb > 256) return false;
    if (reinterpret_cast<std::uintptr_t>(a.kv) % 16 || reinterpret_cast<std::uintptr_t>(a.kv_scales) % 16 ||
        reinterpret_cast<std::uintptr_t>(a.q) % 16)
        return false;
    const long long D = a.dim;
    if (a.block_stride % (4 * D) || a.layer_offset % (4 * D) || a.kind_stride % (4 * D)) return false;
    if (mma_i8_smem_bytes(a.dim, a.tpb) > 200 * 1024) return false;
    return (long long)a.max_blocks * (a.block_stride / D) < (1ll << 31);
}

constexpr long long chunk_smem_bytes(int D, int tpb, int elem = 2) {
    return 1024 + (long long)kChunkRing * 2 * (D * elem / 128) * tpb * 128;
}

// The F32 pool as rows of D floats, boxes of 32 floats x tpb rows, 128-byte swizzle.
CUtensorMap kv_map_f32(const AttnArgs& a, int D) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(D), cuuint64_t((long long)a.max_blocks * (a.block_stride / D))};
    const cuuint64_t strides[1] = {cuuint64_t(D) * 4};
    const cuuint32_t box[2] = {32, cuuint32_t(a.tpb)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(a.kv), dims,
                                            strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

template <int D, int G>
void run_chunk(const AttnArgs& a, cudaStream_t s) {
    if (a.kv_f16) {
        const int smem = int(chunk_smem_bytes(D, a.tpb));
        TVARA_CUDA(cudaFuncSetAttribute(attn_chunk_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        const CUtensorMap map = kv_map_f16(a, D);
        attn_chunk_kernel<D, G><<<dim3(a.n_chunk, a.hkv), kAttnWarps * 32, smem, s>>>(map, a);
    } else {
        const int smem = int(chunk_smem_bytes(D, a.tpb, 4));
        TVARA_CUDA(cudaFuncSetAttribute(attn_chunk_f32_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        const CUtensorMap map = kv_map_f32(a, D);
        attn_chunk_f32_kernel<D, G><<<dim3(a.n_chunk, a.hkv), kAttnWarps * 32, smem, s>>>(map, a);
    }
}

template <int D>
void run_chunk_g(const AttnArgs& a, cudaStream_t s) {
    switch (a.hq / a.hkv) {
        case 1: run_chunk<D, 1>(a, s); break;
        case 2: run_chunk<D, 2>(a, s); break;
        case 3: run_chunk<D, 3>(a, s); break;
        case 4: run_chunk<D, 4>(a, s); break;
        case 5: run_chunk<D, 5>(a, s); break;
        case 6: run_chunk<D, 6>(a, s); break;
        case 7: run_chunk<D, 7>(a, s); break;
        case 8: run_chunk<D, 8>(a, s); break;
        default: throw std::invalid_argument("chunk attention needs 1..8 query heads per KV head");
    }
}

template <int D, int G>
void run_mma_i8(const AttnArgs& a, dim3 grid, cudaStream_t s) {
    const int smem = int(mma_i8_smem_bytes(D, a.tpb));
    TVARA_CUDA(cudaFuncSetAttribute(attn_mma_i8_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const CUtensorMap map = kv_map_i8(a, D);
    attn_mma_i8_kernel<D, G><<<grid, kAttnWarps * 32, smem, s>>>(map, a);
}

template <int D, typename KV, int G>
constexpr bool xpose_ok() {
    constexpr int LPS = (D * int(sizeof(KV)) / 16) < 32 ? (D * int(sizeof(KV)) / 16) : 32;
    return (G & (G - 1)) == 0 && G <= LPS && (D / LPS) % 2 == 0;
}

template <int D, typename KV>
void run_g(const AttnArgs& a, cudaStream_t s) {
    const int g = a.hq / a.hkv;
    dim3 grid(a.n_work, a.hkv);
    // Each warp stages its blocks' K/V runs in a two-deep shared-memory ring;
    // blocks too large for that use the register-streaming kernel instead.
    const long long chunk = (long long)a.tpb * D * sizeof(KV);
    const long long smem = 128 + (long long)kAttnWarps * kRing * 2 * chunk;
    const bool pipe = smem <= 110 * 1024;
    constexpr bool kMmaShape = std::is_same_v<KV, __half> && (D == 64 || D == 128);
    const bool mma = kMmaShape && mma_ok(a);
    switch (g) {
#define TV_G(N)                                                                  \
    case N:                                                                      \
        if (mma) {                                                               \
            if constexpr (kMmaShape) run_mma<D, N>(a, grid, s);                  \
        } else if (pipe && xpose_ok<D, KV, N>()) {                               \
            if constexpr (xpose_ok<D, KV, N>()) run_xpose<D, KV, N>(a, grid, int(smem), s); \
        } else if (pipe) {                                                       \
            run_pipe<D, KV, N>(a, grid, int(smem), s);                           \
        } else {                                                                 \
            attn_kernel<D, KV, N><<<grid, kAttnWarps * 32, 0, s>>>(a);           \
        }                                                                        \
        break;
        TV_G(1) TV_G(2) TV_G(3) TV_G(4) TV_G(5) TV_G(6) TV_G(7) TV_G(8)
#undef TV_G
        default: throw std::invalid_argument("unsupported query/KV head ratio (1..8)");
    }
}

// int8 pools: the tensor-core kernel where its shape conditions hold, else
// the register-streaming kernel (one 16-byte load per lane and slot, decoded
// with the slot's scale).
template <int D>
void run_g_i8(const AttnArgs& a, cudaStream_t s) {
    dim3 grid(a.n_work, a.hkv);
    constexpr bool kMmaShape = D == 64 || D == 128;
    const bool mma = kMmaShape && mma_i8_ok(a);
    switch (a.hq / a.hkv) {
#define TV_G(N)                                                                        \
    case N:                                                                            \
        if (mma) {                                                                     \
            if constexpr (kMmaShape) run_mma_i8<D, N>(a, grid, s);                     \
        } else {                                                                       \
            attn_kernel<D, signed char, N><<<grid, kAttnWarps * 32, 0, s>>>(a);        \
        }                                                                              \
        break;
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

int attention_chunk_rows(int kv_kind, int dim, int group, int tpb) {
    if (kv_kind > 1 || (dim != 64 && dim != 128) || group < 1 || group > 8 || tpb % 16 || tpb > 256) return 0;
    if (chunk_smem_bytes(dim, tpb, kv_kind == 1 ? 2 : 4) > 200 * 1024) return 0;
    return kAttnWarps * (16 / group);
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.n_chunk > 0) {
        const int kind = a.kv_i8 ? 2 : a.kv_f16 ? 1 : 0;
        const bool addressable = reinterpret_cast<std::uintptr_t>(a.kv) % 16 == 0 &&
                                 (long long)a.max_blocks * (a.block_stride / a.dim) < (1ll << 31);
        if (!attention_chunk_rows(kind, a.dim, a.hq / a.hkv, a.tpb) || !addressable)
            throw std::invalid_argument("chunk attention does not apply to this pool");
        if (a.dim == 64) run_chunk_g<64>(a, s);
        else run_chunk_g<128>(a, s);
        TVARA_LAUNCHED();
    }
    if (a.n_work <= 0) return;
    if (a.kv_i8) {
        if (!a.kv_scales) throw std::invalid_argument("int8 KV needs its scales");
        switch (a.dim) {
            case 16: run_g_i8<16>(a, s); break;
            case 32: run_g_i8<32>(a, s); break;
            case 64: run_g_i8<64>(a, s); break;
            case 128: run_g_i8<128>(a, s); break;
            case 256: run_g_i8<256>(a, s); break;
            default: throw std::invalid_argument("unsupported head_dim (16, 32, 64, 128, 256)");
        }
    } else if (a.kv_f16) {
        run_d<__half>(a, s);
    } else {
        run_d<float>(a, s);
    }
    TVARA_LAUNCHED();
    if (a.n_combine > 0) {
        combine_kernel<<<dim3(a.n_combine, a.hq), 128, 0, s>>>(a);
        TVARA_LAUNCHED();
    }
}

}  // namespace tvara
