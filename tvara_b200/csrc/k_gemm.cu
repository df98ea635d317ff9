// Projection for larger token counts on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, activations fed by TMA).
//
// D[w_row][token] = sum_k W[w_row][k] * X[token][k] for a tile of 128 weight
// rows (the MMA's M) and up to 256 tokens (N).  The weight operand comes from
// exact FP16 planes built at load, or from packed rows dequantised by
// producer warps into the UMMA shared-memory layout.
// Precision: the reference multiplies F32 weights by F32 activations
// (core/include/tvara/quant.hpp:163-169); a single FP16 rounding of either
// operand costs ~5e-4 relative per product, which measurably exceeds the 2e-3
// logit budget on deep models.  So both operands are split exactly into
// hi + lo FP16 parts (after an exact power-of-two scaling that keeps them in
// the normal FP16 range: per weight row for W, per token for X) and each
// K-step issues three MMAs, hi*hi + hi*lo + lo*hi, accumulating in F32 --
// products carry ~2^-22 relative error.
//
// Two kernels share the tile, the stage layout and the epilogue:
// * tc_gemm_persist_kernel (weights with prebuilt FP16 planes, the engine's
//   batched path): persistent, warp-specialised -- a TMA warp streams A
//   (planes) and B (split activations) through the stage ring across tile
//   boundaries, an MMA warp accumulates into one of two TMEM buffers, eight
//   epilogue warps drain the other;
// * tc_gemm_kernel (packed weights, the kernel-level ABI): one CTA per tile;
//   warps 0-7 produce A -- thread (r, h) converts weight row r, K-half h of
//   every step from a register ring of packed blocks -- then run the
//   epilogue; warp 8 allocates TMEM and issues the MMAs.
// Epilogue: TMEM lane == weight row; warps w and w+4 split the token columns.
// All TMA loads are per-CTA loads of this GPU's own memory.  Every mbarrier
// wait is bounded: on timeout the kernel records an error code, waits
// (bounded) for its own TMA copies, frees TMEM and exits.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kernels.cuh"
#include "split.cuh"
#include "tma.cuh"

namespace tvara {
namespace {

constexpr int kBM = 128;          // weight rows per tile (MMA M)
constexpr int kBK = 32;           // K per stage (one 64-byte swizzled row of FP16)
constexpr int kStages = 4;
constexpr int kMaxN = 256;        // tokens per tile (MMA N)
constexpr int kProducerWarps = 8;                // two per scheduler: (row, K-half) per thread
constexpr int kProducers = kProducerWarps * 32;
constexpr int kMmaWarp = kProducerWarps;
constexpr int kThreads = kProducers + 32;
constexpr unsigned kSpinLimit = 1u << 26;
constexpr int kATile = kBM * kBK * 2;      // 8 KB per hi/lo A tile
constexpr int kBTileMax = kMaxN * kBK * 2; // 16 KB per hi/lo B tile
constexpr int kPlanes = -1;                // template TYPE: A from prebuilt FP16 planes by TMA

struct TcArgs {
    DeviceMatrix w;
    const int* x_shift;     // per token: X scaled by 2^x_shift
    float* y;
    int ldy;
    int tokens;
    int n_tile;             // tokens per tile (multiple of 16, <= 256)
    int k_steps;            // kBK-steps per split
    int epilogue;
    int atomic;             // split-K: accumulate with atomics
    unsigned idesc;         // tcgen05 instruction descriptor
    int* err;
};

__device__ __forceinline__ unsigned smem_u32(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(std::uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(std::uint64_t* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false after the limit (or when another role gave up).  The
// single MMA-issuing thread polls without sleeping (try_wait itself suspends
// the thread for a while), the producer warps back off after a while.
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, unsigned parity, volatile int* abort_flag, int* err,
                                          int code, bool backoff = true) {
    for (unsigned i = 0; i < kSpinLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        if (backoff && i > 64) __nanosleep(64);
    }
    *abort_flag = 1;
    atomicExch(err, code);
    return false;
}

__device__ __forceinline__ std::uint64_t smem_desc(const void* tile) {
    // K-major, 64-byte swizzle: 8-row atoms of 64-byte rows stacked every 512 B.
    const std::uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (32ull << 32) | (1ull << 46) | (4ull << 61);
}

__device__ __forceinline__ void mma_f16(unsigned tmem_d, std::uint64_t a, std::uint64_t b, unsigned idesc, int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// A from tensor memory (lane = row, column = 2 K elements, even element in
// the low half), B from shared memory.
__device__ __forceinline__ void mma_f16_ts(unsigned tmem_d, unsigned tmem_a, std::uint64_t b, unsigned idesc, int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(std::uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}


// Byte offset of 16-byte chunk c (0..3) of row r in a [rows][64 B] tile with
// the 64-byte swizzle (chunk index XOR bits 1-2 of the row).
__device__ __forceinline__ int sw64(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

// 2^e as a float for |e| <= 126 (exact; used to apply the power-of-two scales).
__device__ __forceinline__ float pow2(int e) { return __uint_as_float(unsigned(127 + e) << 23); }


// ---------------------------------------------------------------- producer
// Packed weights of one row for HALF of a 32-element K-step (hf = 0 or 1),
// fetched ahead of use.  Q4 types: bytes hf*8..hf*8+7 of the 16-byte unit,
// i.e. elements {hf*8..hf*8+7} (low nibbles) and {16+hf*8..} (high nibbles);
// other types: elements hf*16..hf*16+15.
template <int TYPE>
struct Raw;
template <>
struct Raw<kQ4_K> {
    uint2 q;
    uint4 m;  // the block header {d, dmin, scales[12]}
};
template <>
struct Raw<kQ4_0> {
    uint2 q;
    unsigned short d;
};
template <>
struct Raw<kQ8_0> {
    uint4 q;
    unsigned short d;
};
template <>
struct Raw<kF16> {
    uint4 q[2];
};
template <>
struct Raw<kF32> {
    uint4 q[4];
};
template <int TYPE>
struct Ring {  // K-steps of weights kept in flight per producer thread
    static constexpr int kDepth = TYPE == kF32 ? 2 : 4;
};
// 16-byte chunks (of the 64-byte swizzled row) holding v[0..7] and v[8..15]
template <int TYPE>
__device__ __forceinline__ int chunk_a(int hf) { return (TYPE == kQ4_K || TYPE == kQ4_0) ? hf : 2 * hf; }
template <int TYPE>
__device__ __forceinline__ int chunk_b(int hf) { return (TYPE == kQ4_K || TYPE == kQ4_0) ? 2 + hf : 2 * hf + 1; }

template <int TYPE>
__device__ __forceinline__ Raw<TYPE> fetch(const DeviceMatrix& w, long long row, int k0, int hf, bool live) {
    Raw<TYPE> r{};
    if (!live) return r;
    const unsigned char* qs = w.qs + row * w.qs_row;
    const unsigned char* meta = w.meta + row * w.meta_row;
    if constexpr (TYPE == kQ4_K) {
        r.q = __ldg(reinterpret_cast<const uint2*>(qs + (k0 / 32) * 16 + hf * 8));
        r.m = __ldg(reinterpret_cast<const uint4*>(meta + (k0 / 256) * 16));
    } else if constexpr (TYPE == kQ4_0) {
        r.q = __ldg(reinterpret_cast<const uint2*>(qs + (k0 / 32) * 16 + hf * 8));
        r.d = __ldg(reinterpret_cast<const unsigned short*>(meta) + k0 / 32);
    } else if constexpr (TYPE == kQ8_0) {
        r.q = __ldg(reinterpret_cast<const uint4*>(qs + k0 + hf * 16));
        r.d = __ldg(reinterpret_cast<const unsigned short*>(meta) + k0 / 32);
    } else if constexpr (TYPE == kF16) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
            r.q[c] = __ldg(reinterpret_cast<const uint4*>(qs + std::size_t(k0 + hf * 16) * 2) + c);
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            r.q[c] = __ldg(reinterpret_cast<const uint4*>(qs + std::size_t(k0 + hf * 16) * 4) + c);
    }
    return r;
}

__device__ __forceinline__ float h2f(unsigned short h) { return __half2float(__ushort_as_half(h)); }

// Byte k of w placed in the mantissa of 2^23: the float 2^23 + byte.
__device__ __forceinline__ float magic_byte(unsigned w, int k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | unsigned(k)));
}

// The half-step's 16 weights, times 2^shift (exact), into v[16] in the order
// of chunk_a (v[0..7]) then chunk_b (v[8..15]).
template <int TYPE>
__device__ __forceinline__ void convert(const Raw<TYPE>& r, int k0, float scale, float (&v)[16]) {
    if constexpr (TYPE == kQ4_K || TYPE == kQ4_0) {
        float a, b;  // value = a*q - b, already scaled
        if constexpr (TYPE == kQ4_K) {
            const float d = h2f((unsigned short)(r.m.x & 0xffff)), dmin = h2f((unsigned short)(r.m.x >> 16));
            const int g = (k0 / 32) % 8;
            // byte j (0..11) of the packed scales, selected without an indexed array
            auto sbyte = [&](int j) {
                const unsigned word = j < 4 ? r.m.y : j < 8 ? r.m.z : r.m.w;
                return (word >> (8 * (j & 3))) & 255u;
            };
            unsigned sc, mn;
            if (g < 4) {
                sc = sbyte(g) & 63u;
                mn = sbyte(g + 4) & 63u;
            } else {
                sc = (sbyte(g + 4) & 15u) | ((sbyte(g - 4) >> 6) << 4);
                mn = (sbyte(g + 4) >> 4) | ((sbyte(g) >> 6) << 4);
            }
            // small integers to float through the 2^23 magic (no conversion unit)
            a = d * (__uint_as_float(0x4B000000u | sc) - 8388608.f) * scale;
            b = dmin * (__uint_as_float(0x4B000000u | mn) - 8388608.f) * scale;
        } else {
            a = h2f(r.d) * scale;
            b = 8.f * a;
        }
        const unsigned ws[2] = {r.q.x, r.q.y};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const unsigned lo = ws[i] & 0x0F0F0F0Fu, hi = (ws[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[4 * i + k] = fmaf(a, magic_byte(lo, k) - 8388608.f, -b);
                v[8 + 4 * i + k] = fmaf(a, magic_byte(hi, k) - 8388608.f, -b);
            }
        }
    } else if constexpr (TYPE == kQ8_0) {
        const float d = h2f(r.d) * scale;
        const unsigned ws[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const unsigned u = ws[i] ^ 0x80808080u;  // int8 -> biased byte
#pragma unroll
            for (int k = 0; k < 4; ++k) v[4 * i + k] = d * (magic_byte(u, k) - 8388736.f);
        }
    } else if constexpr (TYPE == kF16) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const __half2* h = reinterpret_cast<const __half2*>(&r.q[c]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h[j]);
                v[c * 8 + 2 * j] = f.x * scale;
                v[c * 8 + 2 * j + 1] = f.y * scale;
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            v[c * 4] = __uint_as_float(r.q[c].x) * scale;
            v[c * 4 + 1] = __uint_as_float(r.q[c].y) * scale;
            v[c * 4 + 2] = __uint_as_float(r.q[c].z) * scale;
            v[c * 4 + 3] = __uint_as_float(r.q[c].w) * scale;
        }
    }
}

// a / b for b in [1, 2] without the IEEE division's out-of-line path: the
// approximate quotient corrected once by the exact residual (within about
// half an ulp of the correctly rounded quotient).
__device__ __forceinline__ float div_12(float a, float b) {
    const float q = __fdividef(a, b);
    return __fmaf_rn(__fmaf_rn(-q, b, a), __fdividef(1.f, b), q);
}
// swiglu with div_12 (the epilogue of the Q4_K kernel, where the division's
// call and spills stalled the MMAs)
__device__ __forceinline__ float swiglu_12(float g, float up) {
    const float small = expf(-fabsf(g));
    const float sig = g >= 0.f ? div_12(1.f, 1.f + small) : div_12(small, 1.f + small);
    return __fmul_rn(g, __fmul_rn(sig, up));
}

__device__ __forceinline__ float swiglu(float g, float up) {
    const float small = expf(-fabsf(g));
    const float sig = g >= 0.f ? 1.f / (1.f + small) : small / (1.f + small);
    return __fmul_rn(g, __fmul_rn(sig, up));
}

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                   const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo, TcArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned carve-up: per stage A_hi, A_lo (8 KB each), B_hi, B_lo
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int b_bytes = a.n_tile * kBK * 2;
    const int stage_bytes = 2 * kATile + 2 * kBTileMax;
    unsigned char* stages = base;
    std::uint64_t* full_a = reinterpret_cast<std::uint64_t*>(base + kStages * stage_bytes);  // producers
    std::uint64_t* full_b = full_a + kStages;  // TMA bytes of the X tiles
    std::uint64_t* empty = full_b + kStages;   // MMA finished reading the stage
    std::uint64_t* done = empty + kStages;     // accumulator complete
    unsigned* tmem_slot = reinterpret_cast<unsigned*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // token tiles of one row tile are neighbours in launch order (they share
    // the weight rows in L2)
    const int row0 = blockIdx.y * kBM;
    const int tok0 = blockIdx.x * a.n_tile;
    const int kstep0 = blockIdx.z * a.k_steps;
    const unsigned tmem_cols = a.n_tile <= 32 ? 32 : a.n_tile <= 64 ? 64 : a.n_tile <= 128 ? 128 : 256;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_a[s], kProducers);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const unsigned tmem = *tmem_slot;

    if (warp < kProducerWarps) {
        // ---------------- producers: A tiles (and thread 0: B tiles by TMA).
        // Thread (r, hf): weight row r of the tile, K-half hf of each step.
        const int r = threadIdx.x % kBM;
        const int hf = threadIdx.x / kBM;
        const long long row = row0 + r;
        const bool live = row < a.w.rows;
        const int shift = live ? a.w.row_shift[row] : 0;
        const float scale = pow2(shift);
        // per stage: whether this thread issued a TMA there, and its phase
        unsigned tma_issued = 0, tma_phase = 0;
        if constexpr (TYPE == kPlanes) {
            // A and B tiles both arrive by TMA, issued by lane 0 of warp 0; the
            // whole warp runs the loop so the issuing lane never shares its warp
            // with lanes spinning elsewhere.
            if (warp == 0) {
                for (int ks = 0; ks < a.k_steps; ++ks) {
                    int go = 1;
                    if (lane == 0) {
                        const int s = ks % kStages;
                        const unsigned ph = (ks / kStages) & 1;
                        const int k0 = (kstep0 + ks) * kBK;
                        go = !*abort_flag && mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err, 11, false);
                        if (go) {
                            unsigned char* st = stages + s * stage_bytes;
                            const unsigned bar = smem_u32(&full_b[s]);
                            mbar_expect_tx(&full_b[s], 2 * kATile + 2 * b_bytes);
                            tma_load_2d(smem_u32(st), &map_ahi, k0, row0, bar);
                            tma_load_2d(smem_u32(st + kATile), &map_alo, k0, row0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile), &map_hi, k0, tok0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile + kBTileMax), &map_lo, k0, tok0, bar);
                            tma_issued |= 1u << s;
                            tma_phase = (tma_phase & ~(1u << s)) | (ph << s);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, go, 0)) break;
                }
            }
        } else {
            constexpr int P = Ring<TYPE>::kDepth;
            Raw<TYPE> ring[P];
    #pragma unroll
            for (int j = 0; j < P; ++j)
                ring[j] = fetch<TYPE>(a.w, row, (kstep0 + j) * kBK, hf, live && j < a.k_steps);
            // The K loop is unrolled by the ring depth so every ring slot is a
            // fixed register set (no shifting).
            bool stop = false;
            for (int ks0 = 0; ks0 < a.k_steps && !stop; ks0 += P) {
    #pragma unroll
                for (int j = 0; j < P; ++j) {
                    const int ks = ks0 + j;
                    if (ks >= a.k_steps || *abort_flag) {
                        stop = true;
                        break;
                    }
                    const int s = ks % kStages;
                    const unsigned ph = (ks / kStages) & 1;
                    const int k0 = (kstep0 + ks) * kBK;
                    const Raw<TYPE> cur = ring[j];
                    ring[j] = fetch<TYPE>(a.w, row, k0 + P * kBK, hf, live && ks + P < a.k_steps);
                    float v[16];
                    convert<TYPE>(cur, k0, scale, v);
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err, 11)) {
                        stop = true;
                        break;
                    }
                    unsigned char* st = stages + s * stage_bytes;
                    if (threadIdx.x == 0) {
                        mbar_expect_tx(&full_b[s], 2 * b_bytes);
                        tma_load_2d(smem_u32(st + 2 * kATile), &map_hi, k0, tok0, smem_u32(&full_b[s]));
                        tma_load_2d(smem_u32(st + 2 * kATile + kBTileMax), &map_lo, k0, tok0, smem_u32(&full_b[s]));
                        tma_issued |= 1u << s;
                        tma_phase = (tma_phase & ~(1u << s)) | (ph << s);
                    }
                    unsigned char* ahi = st;
                    unsigned char* alo = st + kATile;
    #pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint4 hi, lo;
                        unsigned* hp = reinterpret_cast<unsigned*>(&hi);
                        unsigned* lp = reinterpret_cast<unsigned*>(&lo);
    #pragma unroll
                        for (int e = 0; e < 4; ++e) split_exact(v[c * 8 + 2 * e], v[c * 8 + 2 * e + 1], hp[e], lp[e]);
                        const int chunk = c == 0 ? chunk_a<TYPE>(hf) : chunk_b<TYPE>(hf);
                        *reinterpret_cast<uint4*>(ahi + sw64(r, chunk)) = hi;
                        *reinterpret_cast<uint4*>(alo + sw64(r, chunk)) = lo;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(&full_a[s]);
                }
            }
        }
        // ---------------- epilogue: TMEM lane r holds weight row row0 + r;
        // warps w and w+4 share lanes 32*(w%4).. and split the token columns
        const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, a.err, 12) ? 1 : 0);
        if (ok) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const float wscale = pow2(-shift);
            for (int c0 = hf * 32; c0 < a.n_tile; c0 += 64) {
                unsigned u[32];
                const unsigned taddr = tmem + ((unsigned)((warp % 4) * 32) << 16) + (unsigned)c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                      "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                      "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
                      "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
                      "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = tok0 + c0 + j;
                    if (c0 + j >= a.n_tile) break;
                    float val = 0.f;
                    if (t < a.tokens) val = __uint_as_float(u[j]) * wscale * pow2(-a.x_shift[t]);
                    if (a.epilogue == kSwiGLU) {
                        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
                        if (t < a.tokens && live && !(r & 1))
                            a.y[(long long)t * a.ldy + row / 2] = swiglu(val, partner);
                    } else if (t < a.tokens && live) {
                        float* dst = a.y + (long long)t * a.ldy + row;
                        if (a.atomic) atomicAdd(dst, val);
                        else if (a.epilogue == kAdd) *dst += val;
                        else *dst = val;
                    }
                }
            }
        }
        // before leaving, every TMA copy this thread issued must have landed
        // (normally long since consumed; after an abort, wait with a bound)
        if (threadIdx.x == 0) {
            for (int s = 0; s < kStages; ++s)
                if (tma_issued >> s & 1u)
                    for (unsigned i = 0; i < kSpinLimit && !mbar_try(&full_b[s], (tma_phase >> s) & 1u); ++i) {
                    }
        }
    } else if (lane == 0) {
        // ---------------- MMA issuer
        const int sub = kBK / 16;
        for (int ks = 0; ks < a.k_steps; ++ks) {
            const int s = ks % kStages;
            const unsigned ph = (ks / kStages) & 1;
            if (!mbar_wait(&full_b[s], ph, abort_flag, a.err, 13, false)) break;
            if (TYPE != kPlanes && !mbar_wait(&full_a[s], ph, abort_flag, a.err, 14, false)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            unsigned char* st = stages + s * stage_bytes;
            const std::uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
            const std::uint64_t bhi = smem_desc(st + 2 * kATile), blo = smem_desc(st + 2 * kATile + kBTileMax);
#pragma unroll
            for (int kk = 0; kk < sub; ++kk) {
                const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;  // 16 K of FP16 = 32 B
                mma_f16(tmem, ahi + adv, bhi + adv, a.idesc, ks > 0 || kk > 0);
                mma_f16(tmem, ahi + adv, blo + adv, a.idesc, 1);
                mma_f16(tmem, alo + adv, bhi + adv, a.idesc, 1);
            }
            mma_commit(&empty[s]);
        }
        mma_commit(done);
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols));
    }
}

// ---------------------------------------------------------------------------
// Persistent variant for prebuilt weight planes: one CTA per SM walks the
// tiles b, b + G, b + 2G, ... (token tiles of a row tile adjacent).  Warp 9
// issues the TMA loads of A (planes) and B (activations) through one stage
// ring that runs on across tile boundaries, warp 8 issues the MMAs into one
// of two TMEM accumulators (2 x 256 columns), and warps 0-7 run the epilogue
// of tile i while the MMAs of tile i+1 proceed -- the epilogue and the
// pipeline fill of each tile are hidden.
constexpr int kPersistThreads = 320;
constexpr int kEpilogueWarps = 8;
constexpr int kMmaWarpP = 8;
constexpr int kTmaWarpP = 9;

struct TileSpace {
    int token_tiles, row_tiles, splits, n_tiles;
};

// row_unit: weight rows per tile (kBM; two kBM halves in the CTA-pair form)
__device__ __forceinline__ void tile_coords(const TileSpace& ts, int t, int n_tile, int k_steps, int& row0, int& tok0,
                                            int& kstep0, int row_unit = kBM) {
    const int tt = t % ts.token_tiles;
    const int rest = t / ts.token_tiles;
    row0 = (rest % ts.row_tiles) * row_unit;
    tok0 = tt * n_tile;
    kstep0 = (rest / ts.row_tiles) * k_steps;
}

__global__ void __launch_bounds__(kPersistThreads, 1)
    tc_gemm_persist_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                           const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                           TcArgs a, TileSpace ts) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int b_bytes = a.n_tile * kBK * 2;
    const int stage_bytes = 2 * kATile + 2 * kBTileMax;
    unsigned char* stages = base;
    std::uint64_t* full = reinterpret_cast<std::uint64_t*>(base + kStages * stage_bytes);  // TMA bytes landed
    std::uint64_t* empty = full + kStages;       // MMA finished reading the stage
    std::uint64_t* acc_full = empty + kStages;   // [2] accumulator ready for the epilogue
    std::uint64_t* acc_empty = acc_full + 2;     // [2] epilogue finished reading it
    unsigned* tmem_slot = reinterpret_cast<unsigned*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpilogueWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarpP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const unsigned tmem = *tmem_slot;

    if (warp == kTmaWarpP) {
        // ---------------- TMA producer (lane 0 issues; the warp stays converged)
        unsigned tma_issued = 0, tma_phase = 0;
        int q = 0;  // K-steps issued by this CTA (stage ring position)
        bool go = true;
        for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
            int row0, tok0, kstep0;
            tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
            for (int ks = 0; ks < a.k_steps; ++ks, ++q) {
                int ok = 1;
                if (lane == 0) {
                    const int s = q % kStages;
                    const unsigned ph = (q / kStages) & 1;
                    const int k0 = (kstep0 + ks) * kBK;
                    ok = !*abort_flag && mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err, 11, false);
                    if (ok) {
                        unsigned char* st = stages + s * stage_bytes;
                        const unsigned bar = smem_u32(&full[s]);
                        mbar_expect_tx(&full[s], 2 * kATile + 2 * b_bytes);
                        tma_load_2d(smem_u32(st), &map_ahi, k0, row0, bar);
                        tma_load_2d(smem_u32(st + kATile), &map_alo, k0, row0, bar);
                        tma_load_2d(smem_u32(st + 2 * kATile), &map_hi, k0, tok0, bar);
                        tma_load_2d(smem_u32(st + 2 * kATile + kBTileMax), &map_lo, k0, tok0, bar);
                        tma_issued |= 1u << s;
                        tma_phase = (tma_phase & ~(1u << s)) | (ph << s);
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    go = false;
                    break;
                }
            }
        }
        // every copy issued must have landed before the CTA leaves
        if (lane == 0)
            for (int s = 0; s < kStages; ++s)
                if (tma_issued >> s & 1u)
                    for (unsigned i = 0; i < kSpinLimit && !mbar_try(&full[s], (tma_phase >> s) & 1u); ++i) {
                    }
    } else if (warp == kMmaWarpP) {
        // ---------------- MMA issuer (lane 0)
        if (lane == 0) {
            int q = 0, i = 0;
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x, ++i) {
                const int b = i & 1;
                if (!mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1, abort_flag, a.err, 15, false)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const unsigned acc = tmem + unsigned(b * 256);
                for (int ks = 0; ks < a.k_steps; ++ks, ++q) {
                    const int s = q % kStages;
                    const unsigned ph = (q / kStages) & 1;
                    if (!mbar_wait(&full[s], ph, abort_flag, a.err, 13, false)) {
                        go = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    unsigned char* st = stages + s * stage_bytes;
                    const std::uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
                    const std::uint64_t bhi = smem_desc(st + 2 * kATile), blo = smem_desc(st + 2 * kATile + kBTileMax);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;  // 16 K of FP16 = 32 B
                        mma_f16(acc, ahi + adv, bhi + adv, a.idesc, ks > 0 || kk > 0);
                        mma_f16(acc, ahi + adv, blo + adv, a.idesc, 1);
                        mma_f16(acc, alo + adv, bhi + adv, a.idesc, 1);
                    }
                    mma_commit(&empty[s]);
                }
                if (go) mma_commit(&acc_full[b]);
            }
        }
    } else {
        // ---------------- epilogue (warps 0-7): TMEM lane r = weight row row0 + r;
        // warps w and w+4 share lanes 32*(w%4).. and split the token columns
        const int r = threadIdx.x % kBM;
        const int hf = threadIdx.x / kBM;
        int i = 0;
        for (int t = blockIdx.x; t < ts.n_tiles; t += gridDim.x, ++i) {
            const int b = i & 1;
            int row0, tok0, kstep0;
            tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (i >> 1) & 1, abort_flag, a.err, 12) ? 1 : 0);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const long long row = row0 + r;
            const bool live = row < a.w.rows;
            const float wscale = pow2(live ? -a.w.row_shift[row] : 0);
            for (int c0 = hf * 32; c0 < a.n_tile; c0 += 64) {
                unsigned u[32];
                const unsigned taddr = tmem + ((unsigned)((warp % 4) * 32) << 16) + unsigned(b * 256 + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                      "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                      "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
                      "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
                      "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int tk = tok0 + c0 + j;
                    if (c0 + j >= a.n_tile) break;
                    float val = 0.f;
                    if (tk < a.tokens) val = __uint_as_float(u[j]) * wscale * pow2(-a.x_shift[tk]);
                    if (a.epilogue == kSwiGLU) {
                        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
                        if (tk < a.tokens && live && !(r & 1))
                            a.y[(long long)tk * a.ldy + row / 2] = swiglu(val, partner);
                    } else if (tk < a.tokens && live) {
                        float* dst = a.y + (long long)tk * a.ldy + row;
                        if (a.atomic) atomicAdd(dst, val);
                        else if (a.epilogue == kAdd) *dst += val;
                        else *dst = val;
                    }
                }
            }
            // this warp is done with the accumulator: release it to the MMA warp
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kMmaWarpP) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---------------------------------------------------------------------------
// Q4_K weights with two MMAs per K-step instead of three (DeviceMatrix::
// qplane).  A Q4_K value is d*sc*q - dmin*m per 32-element sub-block
// (quant.hpp:70-84); sc*q is an integer below 1024, exact in FP16, so the A
// operand is one plane and only the activations are split: P*x_hi + P*x_lo.
// The block scale d changes every 256 elements, so each block's MMAs go to
// one of two 256-column TMEM accumulators and the epilogue warps add
// d[row][block] * accumulator into registers while the MMAs fill the other.
// The min term -sum over sub-blocks of dmin*m * sum(x) is one more block at
// the end of a tile (its first K split only): the exact hi/lo split of
// dmin*m * 2^qmin_shift[row] against the hi/lo split of the sub-block sums
// of x / 32, three MMAs per step over cols/32 columns, scaled back by
// -32 * 2^-qmin_shift[row].  Roles as in the persistent plane kernel: warp 9
// issues the TMA loads through one stage ring, warp 8 the MMAs, warps 0-7
// hold a row and 128 token columns each.
struct Q4kArgs {
    TcArgs t;        // k_steps = 8 * blocks (K-steps per split)
    int blocks;      // 256-element blocks per split
    int min_steps;   // 32-column steps of the min term
};

__global__ void __launch_bounds__(kPersistThreads, 1)
    tc_gemm_q4k_kernel(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                       const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_mhi,
                       const __grid_constant__ CUtensorMap map_mlo, const __grid_constant__ CUtensorMap map_shi,
                       const __grid_constant__ CUtensorMap map_slo, Q4kArgs q, TileSpace ts) {
    const TcArgs& a = q.t;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int b_bytes = a.n_tile * kBK * 2;
    const int stage_bytes = 2 * kATile + 2 * kBTileMax;
    unsigned char* stages = base;
    std::uint64_t* full = reinterpret_cast<std::uint64_t*>(base + kStages * stage_bytes);
    std::uint64_t* empty = full + kStages;
    std::uint64_t* acc_full = empty + kStages;   // [2] block accumulator ready
    std::uint64_t* acc_empty = acc_full + 2;     // [2] epilogue done with it
    unsigned* tmem_slot = reinterpret_cast<unsigned*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = a.w.cols / 256;  // blocks per row

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpilogueWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarpP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const unsigned tmem = *tmem_slot;

    if (warp == kTmaWarpP) {
        unsigned tma_issued = 0, tma_phase = 0;
        int qq = 0;
        bool go = true;
        for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
            int row0, tok0, kstep0;
            tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
            const int steps = a.k_steps + (kstep0 == 0 ? q.min_steps : 0);
            for (int ks = 0; ks < steps; ++ks, ++qq) {
                int ok = 1;
                if (lane == 0) {
                    const int s = qq % kStages;
                    const unsigned ph = (qq / kStages) & 1;
                    ok = !*abort_flag && mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err, 11, false);
                    if (ok) {
                        unsigned char* st = stages + s * stage_bytes;
                        const unsigned bar = smem_u32(&full[s]);
                        if (ks < a.k_steps) {
                            const int k0 = (kstep0 + ks) * kBK;
                            mbar_expect_tx(&full[s], kATile + 2 * b_bytes);
                            tma_load_2d(smem_u32(st), &map_q, k0, row0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile), &map_xhi, k0, tok0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile + kBTileMax), &map_xlo, k0, tok0, bar);
                        } else {
                            const int c0 = (ks - a.k_steps) * kBK;
                            mbar_expect_tx(&full[s], 2 * kATile + 2 * b_bytes);
                            tma_load_2d(smem_u32(st), &map_mhi, c0, row0, bar);
                            tma_load_2d(smem_u32(st + kATile), &map_mlo, c0, row0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile), &map_shi, c0, tok0, bar);
                            tma_load_2d(smem_u32(st + 2 * kATile + kBTileMax), &map_slo, c0, tok0, bar);
                        }
                        tma_issued |= 1u << s;
                        tma_phase = (tma_phase & ~(1u << s)) | (ph << s);
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    go = false;
                    break;
                }
            }
        }
        if (lane == 0)
            for (int s = 0; s < kStages; ++s)
                if (tma_issued >> s & 1u)
                    for (unsigned i = 0; i < kSpinLimit && !mbar_try(&full[s], (tma_phase >> s) & 1u); ++i) {
                    }
    } else if (warp == kMmaWarpP) {
        if (lane == 0) {
            int qq = 0, gb = 0;
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
                const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
                for (int j = 0; j < nb && go; ++j, ++gb) {
                    const int b = gb & 1;
                    if (!mbar_wait(&acc_empty[b], ((gb >> 1) & 1) ^ 1, abort_flag, a.err, 15, false)) {
                        go = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const unsigned acc = tmem + unsigned(b * 256);
                    const bool minterm = j == q.blocks;
                    const int n_steps = minterm ? q.min_steps : 256 / kBK;
                    for (int ks = 0; ks < n_steps; ++ks, ++qq) {
                        const int s = qq % kStages;
                        const unsigned ph = (qq / kStages) & 1;
                        if (!mbar_wait(&full[s], ph, abort_flag, a.err, 13, false)) {
                            go = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;");
                        unsigned char* st = stages + s * stage_bytes;
                        const std::uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
                        const std::uint64_t bhi = smem_desc(st + 2 * kATile), blo = smem_desc(st + 2 * kATile + kBTileMax);
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk) {
                            const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;
                            mma_f16(acc, ahi + adv, bhi + adv, a.idesc, ks > 0 || kk > 0);
                            mma_f16(acc, ahi + adv, blo + adv, a.idesc, 1);
                            if (minterm) mma_f16(acc, alo + adv, bhi + adv, a.idesc, 1);
                        }
                        mma_commit(&empty[s]);
                    }
                    if (go) mma_commit(&acc_full[b]);
                }
            }
        }
    } else {
        // epilogue: TMEM lane r = weight row row0 + r; warps w and w+4 share
        // lanes 32*(w%4).. and take token columns [0, 128) and [128, 256)
        const int r = threadIdx.x % kBM;
        const int hf = threadIdx.x / kBM;
        int gb = 0;
        bool go = true;
        for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
            int row0, tok0, kstep0;
            tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
            const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
            const long long row = row0 + r;
            const bool live = row < a.w.rows;
            float acc[128];
#pragma unroll
            for (int c = 0; c < 128; ++c) acc[c] = 0.f;
            // block scales are loaded one block ahead of their accumulator
            const float* qs_row = a.w.qscale + (live ? row : 0) * kblocks + kstep0 / 8;
            const float min_scale = live ? -32.f * pow2(-a.w.qmin_shift[row]) : 0.f;
            float next = live && q.blocks > 0 ? qs_row[0] : 0.f;
            for (int j = 0; j < nb; ++j, ++gb) {
                const int b = gb & 1;
                const float scale = !live ? 0.f : j < q.blocks ? next : min_scale;
                if (live && j + 1 < q.blocks) next = qs_row[j + 1];
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[b], (gb >> 1) & 1, abort_flag, a.err, 12) ? 1 : 0)) {
                    go = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (hf * 128 + c * 32 >= a.n_tile) break;  // warp-uniform
                    unsigned u[32];
                    const unsigned taddr =
                        tmem + ((unsigned)((warp % 4) * 32) << 16) + unsigned(b * 256 + hf * 128 + c * 32);
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                          "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
                          "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
                          "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                        : "r"(taddr));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) acc[c * 32 + jj] = fmaf(scale, __uint_as_float(u[jj]), acc[c * 32 + jj]);
                }
                asm volatile("tcgen05.fence::before_thread_sync;");
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
            }
            if (!go) break;
            // store, 32 token columns at a time (a runtime loop over one
            // compact body: a fully unrolled 128-column store ran from a cold
            // instruction cache): lane l loads token l's shift (broadcast by
            // shuffles); the residual add is a reduction at L2 (one thread per
            // element, so one IEEE addition as y += val)
            for (int c = 0; c < 4; ++c) {
                const int col0 = hf * 128 + c * 32;
                if (col0 >= a.n_tile) break;  // warp-uniform
                float v[32];
                switch (c) {
#define TVARA_TAKE(C)                                        \
    case C:                                                  \
        _Pragma("unroll") for (int jj = 0; jj < 32; ++jj) v[jj] = acc[C * 32 + jj]; \
        break;
                    TVARA_TAKE(0)
                    TVARA_TAKE(1)
                    TVARA_TAKE(2)
                    TVARA_TAKE(3)
#undef TVARA_TAKE
                }
                const int tl = tok0 + col0 + lane;
                const float inv_l = tl < a.tokens ? pow2(-a.x_shift[tl]) : 0.f;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] *= __shfl_sync(0xffffffffu, inv_l, jj);
                const int ncol = min(32, min(a.n_tile - col0, a.tokens - (tok0 + col0)));
                if (a.epilogue == kSwiGLU) {
                    // rows (2i, 2i+1) are (gate_i, up_i) in adjacent lanes: per
                    // column pair the lanes swap values, the even lane finishes
                    // the even column and the odd lane the odd one (compile-time
                    // indices keep v in registers: a runtime index put it in local
                    // memory, which thrashed the small L1 beside the stages)
                    const bool odd = r & 1;
                    float* dst = a.y + (long long)(tok0 + col0 + odd) * a.ldy + row / 2;
#pragma unroll
                    for (int pr = 0; pr < 16; ++pr) {
                        const float pe = __shfl_xor_sync(0xffffffffu, v[2 * pr], 1);
                        const float po = __shfl_xor_sync(0xffffffffu, v[2 * pr + 1], 1);
                        if (live && 2 * pr + odd < ncol) {
                            const float g = odd ? po : v[2 * pr];
                            const float u = odd ? v[2 * pr + 1] : pe;
                            dst[(long long)(2 * pr) * a.ldy] = swiglu_12(g, u);
                        }
                    }
                } else if (live) {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        if (jj >= ncol) break;
                        float* dst = a.y + (long long)(tok0 + col0 + jj) * a.ldy + row;
                        if (a.atomic || a.epilogue == kAdd) atomicAdd(dst, v[jj]);
                        else *dst = v[jj];
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kMmaWarpP) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---------------------------------------------------------------------------
// The same two-MMA Q4_K product without the FP16 plane in memory: the A
// operand sc*q is built in shared memory from the packed rows at every
// K-step.  Roles, by warpgroup (setmaxnreg gives each its own register
// budget: 200 for the epilogue, 64 for the producers, 48 for the rest):
//   warps 0-7   epilogue: TMEM lane = weight row, warps w and w+4 take token
//               columns [0, 128) and [128, 256); each block's accumulator is
//               added with its scale d into registers, the tile stored at the
//               end (as tc_gemm_q4k_kernel);
//   warps 8-11  producers: thread r (0..127) turns weight row r's 16 packed
//               bytes of a K-step into the 64-byte swizzled K-major row the
//               MMA reads -- 1024 + q as FP16 pairs from one byte permute per
//               pair, sc*q = (1024 + q)*sc - 1024*sc from one fused
//               multiply-add per pair, exact because sc*q is an integer below
//               1024 and the fused result is rounded once;
//   warp 12     issues the MMAs; warp 13 the TMA loads of x (and the min-term
//               tiles) into the main stages; warp 14 the TMA loads of the
//               packed codes (128 rows x 16 bytes per K-step; four K-steps a
//               stage in the tensor-memory form) into a ring of its own,
//               ahead of the producers.
// DRAM carries the packed 0.5625 bytes per weight plus about 0.16 bytes of
// side arrays (qsc, qscale, the min-term split) instead of the plane's 2.
// Barriers: full (x tiles landed and the four producer warps arrived; the MMA
// waits), empty (MMAs done with the stage; TMA warp and producers wait),
// pk_full / pk_empty (packed ring), acc_full / acc_empty (block accumulators).
constexpr int kPkStages = 8;
constexpr int kProducerWarpsP = 4;
constexpr int kProducerWarp0 = 8;
constexpr int kMmaWarpQ = 12, kTmaWarpQ = 13, kPkWarpQ = 14;
constexpr int kQ4kpThreads = 512;

// Two forms of the A operand:
//   kTmemA = false: producers write sc*q into the stage's shared-memory A
//     tile (64-byte swizzled K-major rows); 4 stages of A + x tiles.
//   kTmemA = true: producers write sc*q into tensor memory with tcgen05.st
//     (the producer thread's own lane = its weight row, 16 columns per
//     K-step) and the MMAs read A from there, so a shared-memory stage holds
//     only the x_hi / x_lo tiles (24 KB at the 192-token maximum) and the
//     ring can be 8 deep.  The depth is what matters: a stage comes back to
//     the TMA warp only when its MMAs complete, about 1700-2500 cycles after
//     they were issued (measured with clock stamps), and its x tiles take
//     about 1000 cycles more to land from L2, so a 4-deep ring caps the pace
//     at one K-step per ~1000 cycles against ~350 cycles of MMA work at a
//     176-token tile.  Tensor memory: two block accumulators of 192 columns
//     and 8 A slots of 16 columns.  The min term uses the same slots: each
//     32-unit chunk is two ring steps, the first with the rows' qmin_hi as A
//     (times the hi and lo sub-block sums), the second with qmin_lo (times
//     the hi sums); the producers copy those 64-byte rows from global memory
//     into the slot.
// Cluster (CTA-pair) helpers, used by the pair form below.
constexpr int kPairRows = 2 * kBM;

__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the variable at shared::cta address `local` in CTA `rank`
__device__ __forceinline__ unsigned cluster_addr(unsigned local, unsigned rank) {
    unsigned r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// arrival on a barrier of another CTA of the cluster (default semantics, as
// CUTLASS's 2-SM arrivals: an explicit .release.cluster measured ~0.8 us a
// call, and the data it guards -- TMA bytes, tensor-memory stores -- is already
// complete when the arriving thread observed its own barrier)
__device__ __forceinline__ void mbar_arrive_cluster(unsigned cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// wait on a barrier that the other CTA also signals: default (CTA-scope)
// semantics, as CUTLASS's cluster barriers -- what it guards is async-proxy
// data (TMA bytes, MMA completion) or data the signalling thread had already
// observed complete; an explicit .acquire.cluster cost ~0.4 us a wait
__device__ __forceinline__ bool mbar_try_cluster(std::uint64_t* bar, unsigned parity) { return mbar_try(bar, parity); }
// mbar_wait with cluster-scope acquire (arrivals come from the other CTA too)
__device__ __forceinline__ bool mbar_wait_cluster(std::uint64_t* bar, unsigned parity, volatile int* abort_flag,
                                                  int* err, int code, bool backoff = true) {
    for (unsigned i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_cluster(bar, parity)) return true;
        if (*abort_flag) return false;
        if (backoff && i > 64) __nanosleep(64);
    }
    *abort_flag = 1;
    atomicExch(err, code);
    return false;
}
__device__ __forceinline__ void mma_f16_ts_pair(unsigned tmem_d, unsigned tmem_a, std::uint64_t b, unsigned idesc,
                                                int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
// arrives on the barrier at this shared::cta offset in both CTAs once the MMAs issued so far complete
__device__ __forceinline__ void mma_commit_pair(std::uint64_t* bar) {
    const unsigned short both = 3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(both)
        : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <bool kTmemA>
struct Q4kpForm {
    static constexpr int kRing = kTmemA ? 8 : kStages;
    static constexpr int kMaxTok = kTmemA ? 192 : kMaxN;
    static constexpr int kBTile = kMaxTok * kBK * 2;                   // one x_hi or x_lo tile
    static constexpr int kStageBytes = kTmemA ? 2 * kBTile : 2 * kATile + 2 * kBTileMax;
    static constexpr unsigned kAccCols = kTmemA ? 192u : 256u;         // columns per block accumulator
    static constexpr unsigned kACol = 384;                             // first A slot column (TMEM form)
    // packed-code ring: K-steps per stage (TMA box of 16 bytes per step per row), depth
    static constexpr int kPkSteps = kTmemA ? 4 : 1;
    static constexpr int kPkDepth = kTmemA ? 4 : kPkStages;
    static constexpr int kPkBytes = kBM * 16 * kPkSteps;
    // K-steps per barrier stage: every full / empty round trip (wait, arrive
    // or commit, the refill behind it) costs each role a few hundred cycles
    // whatever it covers -- measured on B200, a bare TMA -> MMA ring runs at
    // ~755 cycles per K-step with one K-step per stage, ~517 with two and
    // ~447 with four (352 of MMA work at a 176-token tile) -- so the
    // tensor-memory form synchronises once per four K-steps: two stages over
    // its eight slots; a tile's steps are padded to whole stages.
    static constexpr int kSub = kTmemA ? 4 : 1;
    static constexpr int kStagesB = kRing / kSub;
    static constexpr int kBarrierBytes = 512;
    static constexpr int smem_bytes() {
        return kRing * kStageBytes + kPkDepth * kPkBytes + 1024 + kBarrierBytes;
    }
};
constexpr int kQ4kpTmemMaxN = Q4kpForm<true>::kMaxTok;

// The CTA-pair form's layout.  A stage's x tiles land ~2 us after their TMA
// issue (measured), so the x ring is four stages of four K-steps: per CTA an
// x slot holds only N/2 tokens (12 KB at 192), sixteen slots fit in 192 KB.
// The A ring (sc*q in tensor memory, written by the producers in ~0.6 us a
// stage) stays two stages of four 16-column slots beside two 192-column block
// accumulators.  The two rings have their own full / empty barriers; the
// producers see only the A ring (kRing, kStagesB below).
struct Q4kPairForm {
    static constexpr int kRing = 8;      // A slots
    static constexpr int kRingX = 16;    // x slots
    static constexpr int kMaxTok = 192;
    static constexpr int kBTile = (kMaxTok / 2) * kBK * 2;  // one CTA's x_hi or x_lo tile
    static constexpr int kStageBytes = 2 * kBTile;          // one x slot
    static constexpr unsigned kAccCols = 192u;
    static constexpr unsigned kACol = 384;
    static constexpr int kPkSteps = 4;
    static constexpr int kPkDepth = 4;
    static constexpr int kPkBytes = kBM * 16 * kPkSteps;
    static constexpr int kSub = 4;
    static constexpr int kStagesB = kRing / kSub;   // A stages
    static constexpr int kStagesX = kRingX / kSub;  // x stages
    static constexpr int kBarrierBytes = 512;
    static constexpr int smem_bytes() {
        return kRingX * kStageBytes + kPkDepth * kPkBytes + 1024 + kBarrierBytes;
    }
};
static_assert(2 * Q4kPairForm::kAccCols + 16 * Q4kPairForm::kRing <= 512, "pair form exceeds tensor memory");
constexpr int kQ4kPairMaxN = Q4kPairForm::kMaxTok;

// Producers of the tensor-memory forms (four warps, thread r = weight row
// row0 + row_off + r): per stage of kSub K-steps, sc*q of the four K-steps of
// one packed-ring stage (or the min term's split minima) into the stage's
// tensor-memory slots, then one arrival per warp on the stage's full barrier
// of this CTA (kPair: the slot waits see the other CTA's commits, cluster
// scope).
template <class F, bool kPair>
__device__ __forceinline__ void q4k_tmem_producers(const Q4kArgs& q, const TileSpace& ts, int t_first, int t_step,
                                                   int row_off, unsigned tmem, const unsigned char* pk_ring,
                                                   std::uint64_t* full, std::uint64_t* empty, std::uint64_t* pk_full,
                                                   std::uint64_t* pk_empty, volatile int* abort_flag) {
    const TcArgs& a = q.t;
    constexpr int kSt = F::kRing;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = a.w.cols / 32;
    const int min_ring = 2 * q.min_steps;
    auto wait_for = [&](std::uint64_t* bar, unsigned parity, int code) {
        return kPair ? mbar_wait_cluster(bar, parity, abort_flag, a.err, code) : mbar_wait(bar, parity, abort_flag, a.err, code);
    };
    const int r = threadIdx.x - kProducerWarp0 * 32;
    const unsigned lane_row = (unsigned)((warp % 4) * 32) << 16;
    int qq = 0, pq = 0;
    bool go = true;
    for (int t = t_first; t < ts.n_tiles && go; t += t_step) {
        int row0, tok0, kstep0;
        tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPair ? kPairRows : kBM);
        const int steps = a.k_steps + (kstep0 == 0 ? min_ring : 0);
        const long long row = row0 + row_off + r;
        const bool live = row < a.w.rows;
        const unsigned char* sc_row = a.w.qsc + (live ? row : 0) * (long long)units + kstep0;
        uint2 sc_cur = live ? __ldg(reinterpret_cast<const uint2*>(sc_row)) : make_uint2(0, 0);
        uint2 sc_next = live && a.k_steps > 8 ? __ldg(reinterpret_cast<const uint2*>(sc_row + 8)) : make_uint2(0, 0);
        static_assert(F::kSub == F::kPkSteps, "a stage is one packed-ring stage");
        for (int p = 0; p < steps; p += F::kSub, qq += F::kSub) {
            const bool main = p < a.k_steps;  // main steps come in whole blocks of 8
            const int G = min(F::kSub, steps - p);
            const int bs = (qq / F::kSub) % F::kStagesB;
            // the stage's slots are free once the MMAs of their previous use are done
            if (!__all_sync(0xffffffffu, wait_for(&empty[bs], ((qq / kSt) & 1) ^ 1, 16) ? 1 : 0)) {
                go = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
            if (main) {
                const int ps = pq % F::kPkDepth;
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&pk_full[ps], (pq / F::kPkDepth) & 1, abort_flag, a.err, 17) ? 1 : 0)) {
                    go = false;
                    break;
                }
                if ((p & 7) == 0 && p > 0) {
                    sc_cur = sc_next;
                    sc_next = live && p + 8 < a.k_steps ? __ldg(reinterpret_cast<const uint2*>(sc_row + p + 8))
                                                        : make_uint2(0, 0);
                }
                const unsigned char* pk = pk_ring + ps * F::kPkBytes;
#pragma unroll
                for (int i = 0; i < F::kPkSteps; ++i) {
                    const uint4 w = *reinterpret_cast<const uint4*>(pk + sw64(r, i));
                    const int pi = p + i;
                    const unsigned sc = (((pi & 4) ? sc_cur.y : sc_cur.x) >> (8 * (pi & 3))) & 255u;
                    const __half2 sc2 = __half2half2(__uint2half_rn(sc));
                    const __half2 off2 = __hneg2(__half2half2(__uint2half_rn(1024u * sc)));
                    const unsigned slot = tmem + lane_row + F::kACol + unsigned(((qq + i) % kSt) * 16);
                    const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)      // low nibbles: elements 0..15, high: 16..31
#pragma unroll
                        for (int c = 0; c < 2; ++c) {   // elements 16 hf + 8 c .. + 7: columns 4 (2 hf + c) ..
                            unsigned out[4];
#pragma unroll
                            for (int k = 0; k < 2; ++k) {
                                const unsigned word = words[2 * c + k];
                                const unsigned nib = hf ? (word >> 4) & 0x0F0F0F0Fu : word & 0x0F0F0F0Fu;
                                const unsigned p0 = __byte_perm(nib, 0x64646464u, 0x4140);  // 1024 + q, bytes 0, 1
                                const unsigned p1 = __byte_perm(nib, 0x64646464u, 0x4342);  // bytes 2, 3
                                const __half2 h0 = __hfma2(*reinterpret_cast<const __half2*>(&p0), sc2, off2);
                                const __half2 h1 = __hfma2(*reinterpret_cast<const __half2*>(&p1), sc2, off2);
                                out[2 * k] = *reinterpret_cast<const unsigned*>(&h0);
                                out[2 * k + 1] = *reinterpret_cast<const unsigned*>(&h1);
                            }
                            asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                             slot + unsigned((2 * hf + c) * 4)),
                                         "r"(out[0]), "r"(out[1]), "r"(out[2]), "r"(out[3])
                                         : "memory");
                        }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&pk_empty[ps]);
                ++pq;
            } else {
                // min term: this row's 32 split minima of each chunk (qmin_hi on even
                // min steps, qmin_lo on odd ones) into the slot; zero past the row's units
                for (int i = 0; i < G; ++i) {
                    const int mi = p + i - a.k_steps;
                    const int c0 = (mi >> 1) * kBK;
                    const unsigned short* src = ((mi & 1) ? a.w.qmin_lo : a.w.qmin_hi) + (live ? row : 0) * units;
                    const unsigned slot = tmem + lane_row + F::kACol + unsigned(((qq + i) % kSt) * 16);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 v = live && c0 + 8 * j < units
                                            ? __ldg(reinterpret_cast<const uint4*>(src + c0 + 8 * j))
                                            : make_uint4(0, 0, 0, 0);
                        asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                         slot + unsigned(j * 4)),
                                     "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                                     : "memory");
                    }
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[bs]);
        }
    }
}

// Epilogue of the packed Q4_K kernels (eight warps; TMEM lane r = weight row
// row0 + row_off + r): per block, d times the block accumulator into
// registers (the min term with its own scale), the tile stored at the end.
// kPair: the arrivals that free an accumulator go to rank 0's barrier.
template <unsigned kAccCols, bool kPair>
__device__ __forceinline__ void q4k_epilogue(const Q4kArgs& q, const TileSpace& ts, int t_first, int t_step, int row_off,
                                             unsigned tmem, std::uint64_t* acc_full, std::uint64_t* acc_empty,
                                             volatile int* abort_flag) {
    const TcArgs& a = q.t;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = a.w.cols / 256;
    auto wait_for = [&](std::uint64_t* bar, unsigned parity, int code) {
        return kPair ? mbar_wait_cluster(bar, parity, abort_flag, a.err, code) : mbar_wait(bar, parity, abort_flag, a.err, code);
    };
    // epilogue: TMEM lane r = weight row row0 + r; warps w and w+4 share
    // lanes 32*(w%4).. and take token columns [0, 128) and [128, 256)
    const int r = threadIdx.x % kBM;
    const int hf = threadIdx.x / kBM;
    int gb = 0;
    bool go = true;
    for (int t = t_first; t < ts.n_tiles && go; t += t_step) {
        int row0, tok0, kstep0;
        tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPair ? kPairRows : kBM);
        const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
        const long long row = row0 + row_off + r;
        const bool live = row < a.w.rows;
        float acc[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) acc[c] = 0.f;
        const float* qs_row = a.w.qscale + (live ? row : 0) * kblocks + kstep0 / 8;
        const float min_scale = live ? -32.f * pow2(-a.w.qmin_shift[row]) : 0.f;
        float next = live && q.blocks > 0 ? qs_row[0] : 0.f;
        for (int j = 0; j < nb; ++j, ++gb) {
            const int b = gb & 1;
            const float scale = !live ? 0.f : j < q.blocks ? next : min_scale;
            if (live && j + 1 < q.blocks) next = qs_row[j + 1];
            if (!__all_sync(0xffffffffu, wait_for(&acc_full[b], (gb >> 1) & 1, 12) ? 1 : 0)) {
                go = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (hf * 128 + c * 32 >= a.n_tile) break;  // warp-uniform
                unsigned u[32];
                const unsigned taddr =
                    tmem + ((unsigned)((warp % 4) * 32) << 16) + unsigned(b) * kAccCols + unsigned(hf * 128 + c * 32);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                      "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                      "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]),
                      "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]),
                      "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) acc[c * 32 + jj] = fmaf(scale, __uint_as_float(u[jj]), acc[c * 32 + jj]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) {
                if (kPair) mbar_arrive_cluster(cluster_addr(smem_u32(&acc_empty[b]), 0));
                else mbar_arrive(&acc_empty[b]);
            }
        }
        if (!go) break;
        // store, 32 token columns at a time (as tc_gemm_q4k_kernel)
        for (int c = 0; c < 4; ++c) {
            const int col0 = hf * 128 + c * 32;
            if (col0 >= a.n_tile) break;  // warp-uniform
            float v[32];
            switch (c) {
#define TVARA_TAKE(C)                                        \
case C:                                                  \
    _Pragma("unroll") for (int jj = 0; jj < 32; ++jj) v[jj] = acc[C * 32 + jj]; \
    break;
                TVARA_TAKE(0)
                TVARA_TAKE(1)
                TVARA_TAKE(2)
                TVARA_TAKE(3)
#undef TVARA_TAKE
            }
            const int tl = tok0 + col0 + lane;
            const float inv_l = tl < a.tokens ? pow2(-a.x_shift[tl]) : 0.f;
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] *= __shfl_sync(0xffffffffu, inv_l, jj);
            const int ncol = min(32, min(a.n_tile - col0, a.tokens - (tok0 + col0)));
            if (a.epilogue == kSwiGLU) {
                const bool odd = r & 1;
                float* dst = a.y + (long long)(tok0 + col0 + odd) * a.ldy + row / 2;
#pragma unroll
                for (int pr = 0; pr < 16; ++pr) {
                    const float pe = __shfl_xor_sync(0xffffffffu, v[2 * pr], 1);
                    const float po = __shfl_xor_sync(0xffffffffu, v[2 * pr + 1], 1);
                    if (live && 2 * pr + odd < ncol) {
                        const float g = odd ? po : v[2 * pr];
                        const float u = odd ? v[2 * pr + 1] : pe;
                        dst[(long long)(2 * pr) * a.ldy] = swiglu_12(g, u);
                    }
                }
            } else if (live) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    if (jj >= ncol) break;
                    float* dst = a.y + (long long)(tok0 + col0 + jj) * a.ldy + row;
                    if (a.atomic || a.epilogue == kAdd) atomicAdd(dst, v[jj]);
                    else *dst = v[jj];
                }
            }
        }
    }
}


template <bool kTmemA, class F = Q4kpForm<kTmemA>>
__global__ void __launch_bounds__(kQ4kpThreads, 1)
    tc_gemm_q4kp_kernel(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                        const __grid_constant__ CUtensorMap map_pk, const __grid_constant__ CUtensorMap map_mhi,
                        const __grid_constant__ CUtensorMap map_mlo, const __grid_constant__ CUtensorMap map_shi,
                        const __grid_constant__ CUtensorMap map_slo, Q4kArgs q, TileSpace ts) {
    const TcArgs& a = q.t;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    constexpr int kSt = F::kRing;
    const int b_bytes = a.n_tile * kBK * 2;
    const int stage_bytes = F::kStageBytes;
    unsigned char* stages = base;
    unsigned char* pk_ring = base + kSt * stage_bytes;
    std::uint64_t* full = reinterpret_cast<std::uint64_t*>(pk_ring + F::kPkDepth * F::kPkBytes);
    std::uint64_t* empty = full + kSt;
    std::uint64_t* pk_full = empty + kSt;
    std::uint64_t* pk_empty = pk_full + F::kPkDepth;
    std::uint64_t* acc_full = pk_empty + F::kPkDepth;  // [2] block accumulator ready
    std::uint64_t* acc_empty = acc_full + 2;         // [2] epilogue done with it
    unsigned* tmem_slot = reinterpret_cast<unsigned*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = a.w.cols / 256;  // blocks per row
    const int units = a.w.cols / 32;     // sub-blocks per row
    constexpr unsigned kAccCols = F::kAccCols;
    // operand tiles of a stage: A (shared-memory form only) and x
    auto tile_bhi = [&](unsigned char* st) { return kTmemA ? st : st + 2 * kATile; };
    auto tile_blo = [&](unsigned char* st) { return kTmemA ? st + F::kBTile : st + 2 * kATile + kBTileMax; };
    // ring steps of a tile's min term: TMEM form two per 32-unit chunk
    const int min_ring = kTmemA ? 2 * q.min_steps : q.min_steps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < F::kStagesB; ++s) {
            mbar_init(&full[s], 1 + kProducerWarpsP);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < F::kPkDepth; ++s) {
            mbar_init(&pk_full[s], 1);
            mbar_init(&pk_empty[s], kProducerWarpsP);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpilogueWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarpQ) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const unsigned tmem = *tmem_slot;

    if (warp >= kMmaWarpQ) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 48;");
        if (kTmemA && warp == kTmaWarpQ) {
            // TMA warp, tensor-memory form: the x tiles of a whole stage (kSub
            // K-steps) under one expect_tx; min-term steps load the sub-block
            // sums (hi; and lo on the qmin_hi steps)
            unsigned issued = 0, phase = 0;
            int qq = 0;  // ring slot of the stage's first K-step (a multiple of kSub)
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
                const int steps = a.k_steps + (kstep0 == 0 ? min_ring : 0);
                for (int p0 = 0; p0 < steps && go; p0 += F::kSub, qq += F::kSub) {
                    int ok = 1;
                    if (lane == 0) {
                        const int bs = (qq / F::kSub) % F::kStagesB;
                        const unsigned ph = (qq / kSt) & 1;
                        ok = !*abort_flag && mbar_wait(&empty[bs], ph ^ 1, abort_flag, a.err, 11, false);
                        if (ok) {
                            const int n = min(F::kSub, steps - p0);
                            unsigned bytes = 0;
                            for (int i = 0; i < n; ++i) {
                                const int p = p0 + i;
                                bytes += unsigned(p < a.k_steps || !((p - a.k_steps) & 1) ? 2 : 1) * unsigned(b_bytes);
                            }
                            mbar_expect_tx(&full[bs], bytes);
                            const unsigned bar = smem_u32(&full[bs]);
                            for (int i = 0; i < n; ++i) {
                                const int p = p0 + i;
                                unsigned char* st = stages + ((qq + i) % kSt) * stage_bytes;
                                if (p < a.k_steps) {
                                    const int k0 = (kstep0 + p) * kBK;
                                    tma_load_2d(smem_u32(tile_bhi(st)), &map_xhi, k0, tok0, bar);
                                    tma_load_2d(smem_u32(tile_blo(st)), &map_xlo, k0, tok0, bar);
                                } else {
                                    const int mi = p - a.k_steps;
                                    const int c0 = (mi >> 1) * kBK;
                                    tma_load_2d(smem_u32(tile_bhi(st)), &map_shi, c0, tok0, bar);
                                    if (!(mi & 1)) tma_load_2d(smem_u32(tile_blo(st)), &map_slo, c0, tok0, bar);
                                }
                            }
                            issued |= 1u << bs;
                            phase = (phase & ~(1u << bs)) | (ph << bs);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, ok, 0)) go = false;
                }
            }
            if (lane == 0)
                for (int bs = 0; bs < F::kStagesB; ++bs)
                    if (issued >> bs & 1u)
                        for (unsigned i = 0; i < kSpinLimit && !mbar_try(&full[bs], (phase >> bs) & 1u); ++i) {
                        }
        } else if (warp == kTmaWarpQ || warp == kPkWarpQ) {
            // TMA warp: x tiles (and the min-term tiles) into the main stages;
            // packed warp: the packed codes of the production steps into its ring
            const bool pk = warp == kPkWarpQ;
            unsigned issued = 0, phase = 0;
            int qq = 0;
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
                const int steps = pk ? a.k_steps / F::kPkSteps : a.k_steps + (kstep0 == 0 ? min_ring : 0);
                for (int ks = 0; ks < steps; ++ks, ++qq) {
                    int ok = 1;
                    if (lane == 0) {
                        const int ring = pk ? F::kPkDepth : kSt;
                        const int s = qq % ring;
                        const unsigned ph = (qq / ring) & 1;
                        ok = !*abort_flag && mbar_wait(pk ? &pk_empty[s] : &empty[s], ph ^ 1, abort_flag, a.err, 11, false);
                        if (ok && pk) {
                            mbar_expect_tx(&pk_full[s], F::kPkBytes);
                            tma_load_2d(smem_u32(pk_ring + s * F::kPkBytes), &map_pk, (kstep0 + ks * F::kPkSteps) * kBK / 2, row0,
                                        smem_u32(&pk_full[s]));
                        } else if (ok) {
                            unsigned char* st = stages + s * stage_bytes;
                            const unsigned bar = smem_u32(&full[s]);
                            if (ks < a.k_steps) {
                                const int k0 = (kstep0 + ks) * kBK;
                                mbar_expect_tx(&full[s], 2 * b_bytes);
                                tma_load_2d(smem_u32(tile_bhi(st)), &map_xhi, k0, tok0, bar);
                                tma_load_2d(smem_u32(tile_blo(st)), &map_xlo, k0, tok0, bar);
                            } else if (kTmemA) {
                                // min term: sub-block sums of x (hi; and lo on the qmin_hi step)
                                const int mi = ks - a.k_steps;
                                const int c0 = (mi >> 1) * kBK;
                                mbar_expect_tx(&full[s], (mi & 1 ? 1 : 2) * b_bytes);
                                tma_load_2d(smem_u32(tile_bhi(st)), &map_shi, c0, tok0, bar);
                                if (!(mi & 1)) tma_load_2d(smem_u32(tile_blo(st)), &map_slo, c0, tok0, bar);
                            } else {
                                const int c0 = (ks - a.k_steps) * kBK;
                                mbar_expect_tx(&full[s], 2 * kATile + 2 * b_bytes);
                                tma_load_2d(smem_u32(st), &map_mhi, c0, row0, bar);
                                tma_load_2d(smem_u32(st + kATile), &map_mlo, c0, row0, bar);
                                tma_load_2d(smem_u32(tile_bhi(st)), &map_shi, c0, tok0, bar);
                                tma_load_2d(smem_u32(tile_blo(st)), &map_slo, c0, tok0, bar);
                            }
                        }
                        if (ok) {
                            issued |= 1u << s;
                            phase = (phase & ~(1u << s)) | (ph << s);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        go = false;
                        break;
                    }
                }
            }
            if (lane == 0)
                for (int s = 0; s < (pk ? F::kPkDepth : kSt); ++s)
                    if (issued >> s & 1u)
                        for (unsigned i = 0; i < kSpinLimit && !mbar_try(pk ? &pk_full[s] : &full[s], (phase >> s) & 1u);
                             ++i) {
                        }
        } else if (kTmemA && warp == kMmaWarpQ && lane == 0) {
            // MMA thread, tensor-memory form: one full wait and one commit per
            // stage; a main block (8 K-steps) is two stages, the min block
            // ceil(min_ring / kSub) (the last one padded)
            int qq = 0, gb = 0;
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
                const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
                for (int j = 0; j < nb && go; ++j, ++gb) {
                    const int b = gb & 1;
                    if (!mbar_wait(&acc_empty[b], ((gb >> 1) & 1) ^ 1, abort_flag, a.err, 15, false)) {
                        go = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const unsigned acc = tmem + unsigned(b) * kAccCols;
                    const bool minterm = j == q.blocks;
                    const int n_steps = minterm ? min_ring : 256 / kBK;
                    for (int p0 = 0; p0 < n_steps; p0 += F::kSub, qq += F::kSub) {
                        const int bs = (qq / F::kSub) % F::kStagesB;
                        if (!mbar_wait(&full[bs], (qq / kSt) & 1, abort_flag, a.err, 13, false)) {
                            go = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;");
                        const int n = min(F::kSub, n_steps - p0);
                        for (int i = 0; i < n; ++i) {
                            const int ks = p0 + i;  // K-step within the block
                            const int s = (qq + i) % kSt;
                            unsigned char* st = stages + s * stage_bytes;
                            const std::uint64_t bhi = smem_desc(tile_bhi(st)), blo = smem_desc(tile_blo(st));
                            // A from the slot: 8 columns per 16 K elements; on the min term's
                            // qmin_lo steps (odd) only the hi sums
                            const unsigned at = tmem + F::kACol + unsigned(s * 16);
                            const bool two = !minterm || !(ks & 1);
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk) {
                                const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;
                                mma_f16_ts(acc, at + unsigned(kk * 8), bhi + adv, a.idesc, ks > 0 || kk > 0);
                                if (two) mma_f16_ts(acc, at + unsigned(kk * 8), blo + adv, a.idesc, 1);
                            }
                        }
                        mma_commit(&empty[bs]);
                    }
                    if (go) mma_commit(&acc_full[b]);
                }
            }
        } else if (warp == kMmaWarpQ && lane == 0) {
            int qq = 0, gb = 0;
            bool go = true;
            for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
                const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
                for (int j = 0; j < nb && go; ++j, ++gb) {
                    const int b = gb & 1;
                    if (!mbar_wait(&acc_empty[b], ((gb >> 1) & 1) ^ 1, abort_flag, a.err, 15, false)) {
                        go = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const unsigned acc = tmem + unsigned(b) * kAccCols;
                    const bool minterm = j == q.blocks;
                    const int n_steps = minterm ? min_ring : 256 / kBK;
                    for (int ks = 0; ks < n_steps; ++ks, ++qq) {
                        const int s = qq % kSt;
                        const unsigned ph = (qq / kSt) & 1;
                        if (!mbar_wait(&full[s], ph, abort_flag, a.err, 13, false)) {
                            go = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;");
                        unsigned char* st = stages + s * stage_bytes;
                        const std::uint64_t bhi = smem_desc(tile_bhi(st)), blo = smem_desc(tile_blo(st));
                        if (kTmemA) {
                            // A from the step's tensor-memory slot: 8 columns per 16 K elements; on
                            // the min term's qmin_lo steps (odd) only the hi sums
                            const unsigned at = tmem + F::kACol + unsigned(s * 16);
                            const bool two = !minterm || !(ks & 1);
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk) {
                                const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;
                                mma_f16_ts(acc, at + unsigned(kk * 8), bhi + adv, a.idesc, ks > 0 || kk > 0);
                                if (two) mma_f16_ts(acc, at + unsigned(kk * 8), blo + adv, a.idesc, 1);
                            }
                        } else {
                            const std::uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk) {
                                const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;
                                mma_f16(acc, ahi + adv, bhi + adv, a.idesc, ks > 0 || kk > 0);
                                mma_f16(acc, ahi + adv, blo + adv, a.idesc, 1);
                                if (minterm) mma_f16(acc, alo + adv, bhi + adv, a.idesc, 1);
                            }
                        }
                        mma_commit(&empty[s]);
                    }
                    if (go) mma_commit(&acc_full[b]);
                }
            }
        }
    } else if (kTmemA && warp >= kProducerWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");
        q4k_tmem_producers<F, false>(q, ts, blockIdx.x, gridDim.x, 0, tmem, pk_ring, full, empty, pk_full, pk_empty, abort_flag);
    } else if (warp >= kProducerWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");
        // producers: thread r = weight row row0 + r, both nibble halves
        const int r = threadIdx.x - kProducerWarp0 * 32;
        int qq = 0, pq = 0;
        bool go = true;
        for (int t = blockIdx.x; t < ts.n_tiles && go; t += gridDim.x) {
            int row0, tok0, kstep0;
            tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0);
            const int steps = a.k_steps + (kstep0 == 0 ? min_ring : 0);
            const long long row = row0 + r;
            const bool live = row < a.w.rows;
            const unsigned char* sc_row = a.w.qsc + (live ? row : 0) * (long long)units + kstep0;
            // sub-block scales of a block (8 bytes), loaded a block ahead
            uint2 sc_cur = live ? __ldg(reinterpret_cast<const uint2*>(sc_row)) : make_uint2(0, 0);
            uint2 sc_next = live && a.k_steps > 8 ? __ldg(reinterpret_cast<const uint2*>(sc_row + 8)) : make_uint2(0, 0);
            for (int p = 0; p < steps; ++p, ++qq) {
                const int s = qq % kSt;
                const unsigned ph = (qq / kSt) & 1;
                // the stage is free once the MMAs of its previous use are done
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err, 16) ? 1 : 0)) {
                    go = false;
                    break;
                }
                if (kTmemA) asm volatile("tcgen05.fence::after_thread_sync;");
                if (p < a.k_steps) {
                    const int ps = pq % F::kPkDepth;
                    const unsigned pph = (pq / F::kPkDepth) & 1;
                    if (!__all_sync(0xffffffffu, mbar_wait(&pk_full[ps], pph, abort_flag, a.err, 17) ? 1 : 0)) {
                        go = false;
                        break;
                    }
                    const uint4 w = *reinterpret_cast<const uint4*>(pk_ring + ps * F::kPkBytes + r * 16);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&pk_empty[ps]);
                    ++pq;
                    if ((p & 7) == 0 && p > 0) {
                        sc_cur = sc_next;
                        sc_next = live && p + 8 < a.k_steps ? __ldg(reinterpret_cast<const uint2*>(sc_row + p + 8))
                                                            : make_uint2(0, 0);
                    }
                    const unsigned sc = (((p & 4) ? sc_cur.y : sc_cur.x) >> (8 * (p & 3))) & 255u;
                    const __half2 sc2 = __half2half2(__uint2half_rn(sc));
                    const __half2 off2 = __hneg2(__half2half2(__uint2half_rn(1024u * sc)));
                    unsigned char* st = stages + s * stage_bytes;
                    const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)      // low nibbles: elements 0..15, high: 16..31
#pragma unroll
                        for (int c = 0; c < 2; ++c) {   // 16-byte chunk 2 hf + c: elements 16 hf + 8 c .. + 7
                            unsigned out[4];
#pragma unroll
                            for (int k = 0; k < 2; ++k) {
                                const unsigned word = words[2 * c + k];
                                const unsigned nib = hf ? (word >> 4) & 0x0F0F0F0Fu : word & 0x0F0F0F0Fu;
                                const unsigned p0 = __byte_perm(nib, 0x64646464u, 0x4140);  // 1024 + q, bytes 0, 1
                                const unsigned p1 = __byte_perm(nib, 0x64646464u, 0x4342);  // bytes 2, 3
                                const __half2 h0 = __hfma2(*reinterpret_cast<const __half2*>(&p0), sc2, off2);
                                const __half2 h1 = __hfma2(*reinterpret_cast<const __half2*>(&p1), sc2, off2);
                                out[2 * k] = *reinterpret_cast<const unsigned*>(&h0);
                                out[2 * k + 1] = *reinterpret_cast<const unsigned*>(&h1);
                            }
                            if (kTmemA) {
                                // elements 8 (2 hf + c) .. + 7: columns 4 (2 hf + c) .. + 3 of the slot
                                const unsigned taddr = tmem + ((unsigned)((warp % 4) * 32) << 16) + F::kACol +
                                                       unsigned(s * 16 + (2 * hf + c) * 4);
                                asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
                                             "r"(out[0]), "r"(out[1]), "r"(out[2]), "r"(out[3])
                                             : "memory");
                            } else {
                                *reinterpret_cast<uint4*>(st + sw64(r, 2 * hf + c)) =
                                    make_uint4(out[0], out[1], out[2], out[3]);
                            }
                        }
                    if (kTmemA) {
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        asm volatile("tcgen05.fence::before_thread_sync;");
                    } else {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    }
                } else if (kTmemA) {
                    // min term: this row's 32 split minima of the chunk (qmin_hi on even
                    // steps, qmin_lo on odd ones) into the slot; zero past the row's units
                    const int mi = p - a.k_steps;
                    const int c0 = (mi >> 1) * kBK;
                    const unsigned short* src = ((mi & 1) ? a.w.qmin_lo : a.w.qmin_hi) + (live ? row : 0) * units;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 v = live && c0 + 8 * j < units
                                            ? __ldg(reinterpret_cast<const uint4*>(src + c0 + 8 * j))
                                            : make_uint4(0, 0, 0, 0);
                        const unsigned taddr =
                            tmem + ((unsigned)((warp % 4) * 32) << 16) + F::kACol + unsigned(s * 16 + j * 4);
                        asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
                                     "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                                     : "memory");
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;");
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 200;");
        q4k_epilogue<kAccCols, false>(q, ts, blockIdx.x, gridDim.x, 0, tmem, acc_full, acc_empty, abort_flag);
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kMmaWarpQ) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---------------------------------------------------------------------------
// The CTA-pair form (tcgen05 cta_group::2): a cluster of two CTAs on the two
// SMs of a TPC computes a 256-row x N-token tile with one M=256 MMA stream.
// CTA rank r holds weight rows [128 r, 128 r + 128) of the tile -- its
// producers build their rows' sc*q into its own tensor memory (same slots and
// lanes as the one-CTA tensor-memory form), its epilogue reads and stores its
// own 128 x N accumulator -- and x tokens [N/2 r, N/2 r + N/2) of the tile in
// its shared memory; the MMAs (issued by rank 0) read A and B from both.  Per
// SM this halves the x bytes streamed from L2 per multiply-add, which is what
// bounds the one-CTA form.  Barriers: each CTA's TMA and producers complete a
// stage on that CTA's own full barrier (plain per-CTA TMA loads; a load that
// completed on the other CTA's barrier measured three times slower per byte);
// rank 1's MMA-warp lane relays its stage completion with one arrival on rank
// 0's full barrier; rank 0's acc_empty collects both epilogues; the commits
// after a stage and after a block arrive on the empty / acc_full barriers of
// both CTAs.  No load uses multicast.
// Measured (B200, 6144 x 4096 x 512 tokens): 1.57 us per stage of four K-steps
// at N = 176 against 0.96 us of MMA issue -- the two-stage A ring waits on the
// cross-CTA round trip (MMA completion -> both CTAs' producers -> relay) --
// 86 us against 67 us for the one-CTA form; a four-stage A ring needs N <= 128
// and is then bound by MMA issue (~100 cycles per M=256 instruction).
// Warp roles as tc_gemm_q4kp_kernel<true> in both CTAs (rank 1's MMA warp
// allocates and frees tensor memory with rank 0's and runs the relay); tiles
// are 256 rows (TileSpace row tiles count pairs of 128-row halves), one per
// cluster at a time.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kQ4kpThreads, 1)
    tc_gemm_q4k2_kernel(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                        const __grid_constant__ CUtensorMap map_pk, const __grid_constant__ CUtensorMap map_shi,
                        const __grid_constant__ CUtensorMap map_slo, Q4kArgs q, TileSpace ts) {
    const TcArgs& a = q.t;
    using F = Q4kPairForm;
    constexpr int kSt = F::kRing;    // A slots (tensor memory)
    constexpr int kSx = F::kRingX;   // x slots (shared memory)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the carve-up must sit at the same shared::cta offsets in both CTAs (the
    // MMA's B descriptors and the commits name one offset for both)
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int half_n = a.n_tile / 2;
    const int b_bytes = a.n_tile * kBK * 2;  // x bytes of one part (hi or lo) of a K-step, both CTAs
    const int stage_bytes = F::kStageBytes;
    unsigned char* stages = base;  // kSx x slots
    unsigned char* pk_ring = base + kSx * stage_bytes;
    std::uint64_t* x_full = reinterpret_cast<std::uint64_t*>(pk_ring + F::kPkDepth * F::kPkBytes);
    std::uint64_t* x_empty = x_full + F::kStagesX;
    std::uint64_t* full = x_empty + F::kStagesX;   // A ring
    std::uint64_t* empty = full + F::kStagesB;
    std::uint64_t* pk_full = empty + F::kStagesB;
    std::uint64_t* pk_empty = pk_full + F::kPkDepth;
    std::uint64_t* acc_full = pk_empty + F::kPkDepth;  // [2] block accumulator ready (this CTA's half)
    std::uint64_t* acc_empty = acc_full + 2;           // [2] rank 0's: both epilogues done with it
    unsigned* tmem_slot = reinterpret_cast<unsigned*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned rank = cluster_rank();
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int kblocks = a.w.cols / 256;
    const int units = a.w.cols / 32;
    constexpr unsigned kAccCols = F::kAccCols;
    const int min_ring = 2 * q.min_steps;
    auto tile_bhi = [&](unsigned char* st) { return st; };
    auto tile_blo = [&](unsigned char* st) { return st + F::kBTile; };

    if (threadIdx.x == 0) {
        // this CTA's TMA (expect_tx) / producer warps; on rank 0 also rank 1's relay
        for (int s = 0; s < F::kStagesX; ++s) {
            mbar_init(&x_full[s], 1 + (rank == 0 ? 1 : 0));
            mbar_init(&x_empty[s], 1);
        }
        for (int s = 0; s < F::kStagesB; ++s) {
            mbar_init(&full[s], kProducerWarpsP + (rank == 0 ? 1 : 0));
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < F::kPkDepth; ++s) {
            mbar_init(&pk_full[s], 1);
            mbar_init(&pk_empty[s], kProducerWarpsP);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * kEpilogueWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarpQ) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival
    asm volatile("tcgen05.fence::after_thread_sync;");
    const unsigned tmem = *tmem_slot;

    if (warp >= kMmaWarpQ) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 48;");
        if (warp == kTmaWarpQ) {
            // x tiles of this CTA's half of the tokens, a stage at a time, on
            // this CTA's own x_full barrier
            unsigned issued = 0, phase = 0;
            int qq = 0;
            bool go = true;
            for (int t = pair; t < ts.n_tiles && go; t += pairs) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPairRows);
                const int steps = a.k_steps + (kstep0 == 0 ? min_ring : 0);
                const int my_tok = tok0 + int(rank) * half_n;
                for (int p0 = 0; p0 < steps && go; p0 += F::kSub, qq += F::kSub) {
                    int ok = 1;
                    if (lane == 0) {
                        const int bs = (qq / F::kSub) % F::kStagesX;
                        const unsigned ph = (qq / kSx) & 1;
                        ok = !*abort_flag && mbar_wait_cluster(&x_empty[bs], ph ^ 1, abort_flag, a.err, 11, false);
                        if (ok) {
                            const int n = min(F::kSub, steps - p0);
                            unsigned bytes = 0;
                            for (int i = 0; i < n; ++i) {
                                const int p = p0 + i;
                                bytes += unsigned(p < a.k_steps || !((p - a.k_steps) & 1) ? 2 : 1) * unsigned(b_bytes / 2);
                            }
                            mbar_expect_tx(&x_full[bs], bytes);
                            const unsigned bar = smem_u32(&x_full[bs]);
                            for (int i = 0; i < n; ++i) {
                                const int p = p0 + i;
                                unsigned char* st = stages + ((qq + i) % kSx) * stage_bytes;
                                if (p < a.k_steps) {
                                    const int k0 = (kstep0 + p) * kBK;
                                    tma_load_2d(smem_u32(tile_bhi(st)), &map_xhi, k0, my_tok, bar);
                                    tma_load_2d(smem_u32(tile_blo(st)), &map_xlo, k0, my_tok, bar);
                                } else {
                                    const int mi = p - a.k_steps;
                                    const int c0 = (mi >> 1) * kBK;
                                    tma_load_2d(smem_u32(tile_bhi(st)), &map_shi, c0, my_tok, bar);
                                    if (!(mi & 1)) tma_load_2d(smem_u32(tile_blo(st)), &map_slo, c0, my_tok, bar);
                                }
                            }
                            issued |= 1u << bs;
                            phase = (phase & ~(1u << bs)) | (ph << bs);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, ok, 0)) go = false;
                }
            }
            if (lane == 0)
                for (int bs = 0; bs < F::kStagesX; ++bs)
                    if (issued >> bs & 1u)
                        for (unsigned i = 0; i < kSpinLimit && !mbar_try_cluster(&x_full[bs], (phase >> bs) & 1u); ++i) {
                        }
        } else if (warp == kPkWarpQ) {
            // packed codes of this CTA's 128 rows into its own ring
            unsigned issued = 0, phase = 0;
            int qq = 0;
            bool go = true;
            for (int t = pair; t < ts.n_tiles && go; t += pairs) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPairRows);
                const int my_row0 = row0 + int(rank) * kBM;
                const int groups = a.k_steps / F::kPkSteps;
                for (int g = 0; g < groups; ++g, ++qq) {
                    int ok = 1;
                    if (lane == 0) {
                        const int s = qq % F::kPkDepth;
                        const unsigned ph = (qq / F::kPkDepth) & 1;
                        ok = !*abort_flag && mbar_wait(&pk_empty[s], ph ^ 1, abort_flag, a.err, 11, false);
                        if (ok) {
                            mbar_expect_tx(&pk_full[s], F::kPkBytes);
                            tma_load_2d(smem_u32(pk_ring + s * F::kPkBytes), &map_pk, (kstep0 + g * F::kPkSteps) * kBK / 2,
                                        my_row0, smem_u32(&pk_full[s]));
                            issued |= 1u << s;
                            phase = (phase & ~(1u << s)) | (ph << s);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        go = false;
                        break;
                    }
                }
            }
            if (lane == 0)
                for (int s = 0; s < F::kPkDepth; ++s)
                    if (issued >> s & 1u)
                        for (unsigned i = 0; i < kSpinLimit && !mbar_try(&pk_full[s], (phase >> s) & 1u); ++i) {
                        }
        } else if (warp == kMmaWarpQ && lane == 0 && rank == 1) {
            // relay: once this CTA's x tiles and A slots of a stage are in place,
            // one arrival on each of rank 0's two full barriers of that stage
            int qq = 0;
            bool go = true;
            for (int t = pair; t < ts.n_tiles && go; t += pairs) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPairRows);
                const int steps = a.k_steps + (kstep0 == 0 ? min_ring : 0);
                for (int p0 = 0; p0 < steps; p0 += F::kSub, qq += F::kSub) {
                    const int xs = (qq / F::kSub) % F::kStagesX, as = (qq / F::kSub) % F::kStagesB;
                    if (!mbar_wait_cluster(&x_full[xs], (qq / kSx) & 1, abort_flag, a.err, 14, false) ||
                        !mbar_wait_cluster(&full[as], (qq / kSt) & 1, abort_flag, a.err, 14, false)) {
                        go = false;
                        break;
                    }
                    mbar_arrive_cluster(cluster_addr(smem_u32(&x_full[xs]), 0));
                    mbar_arrive_cluster(cluster_addr(smem_u32(&full[as]), 0));
                }
            }
        } else if (warp == kMmaWarpQ && lane == 0 && rank == 0) {
            // MMA thread (rank 0): M = 256 over both CTAs' tensor memory
            const unsigned idesc = (a.idesc & ~(31u << 24)) | (unsigned(kPairRows >> 4) << 24);
            int qq = 0, gb = 0;
            bool go = true;
            for (int t = pair; t < ts.n_tiles && go; t += pairs) {
                int row0, tok0, kstep0;
                tile_coords(ts, t, a.n_tile, a.k_steps, row0, tok0, kstep0, kPairRows);
                const int nb = q.blocks + (kstep0 == 0 ? 1 : 0);
                for (int j = 0; j < nb && go; ++j, ++gb) {
                    const int b = gb & 1;
                    if (!mbar_wait_cluster(&acc_empty[b], ((gb >> 1) & 1) ^ 1, abort_flag, a.err, 15, false)) {
                        go = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const unsigned acc = tmem + unsigned(b) * kAccCols;
                    const bool minterm = j == q.blocks;
                    const int n_steps = minterm ? min_ring : 256 / kBK;
                    for (int p0 = 0; p0 < n_steps; p0 += F::kSub, qq += F::kSub) {
                        const int xs = (qq / F::kSub) % F::kStagesX, as = (qq / F::kSub) % F::kStagesB;
                        if (!mbar_wait_cluster(&x_full[xs], (qq / kSx) & 1, abort_flag, a.err, 13, false) ||
                            !mbar_wait_cluster(&full[as], (qq / kSt) & 1, abort_flag, a.err, 13, false)) {
                            go = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;");
                        const int n = min(F::kSub, n_steps - p0);
                        for (int i = 0; i < n; ++i) {
                            const int ks = p0 + i;
                            unsigned char* st = stages + ((qq + i) % kSx) * stage_bytes;
                            const std::uint64_t bhi = smem_desc(tile_bhi(st)), blo = smem_desc(tile_blo(st));
                            const unsigned at = tmem + F::kACol + unsigned(((qq + i) % kSt) * 16);
                            const bool two = !minterm || !(ks & 1);
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk) {
                                const std::uint64_t adv = (std::uint64_t)(kk * 32) >> 4;
                                mma_f16_ts_pair(acc, at + unsigned(kk * 8), bhi + adv, idesc, ks > 0 || kk > 0);
                                if (two) mma_f16_ts_pair(acc, at + unsigned(kk * 8), blo + adv, idesc, 1);
                            }
                        }
                        mma_commit_pair(&x_empty[xs]);
                        mma_commit_pair(&empty[as]);
                    }
                    if (go) mma_commit_pair(&acc_full[b]);
                }
            }
        }
    } else if (warp >= kProducerWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");
        q4k_tmem_producers<Q4kPairForm, true>(q, ts, pair, pairs, int(rank) * kBM, tmem, pk_ring, full, empty, pk_full, pk_empty,
                                 abort_flag);
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 200;");
        q4k_epilogue<kAccCols, true>(q, ts, pair, pairs, int(rank) * kBM, tmem, acc_full, acc_empty, abort_flag);
    }
    // neither CTA leaves (or frees tensor memory) while the other may still
    // read its tensor memory or signal its barriers
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    cluster_sync_all();
    if (warp == kMmaWarpQ) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
    (void)kblocks;
    (void)units;
}

// ---------------------------------------------------------------------------
// Small batches (5 .. 64 tokens) of Q4_K rows on mma.sync, straight from the
// packed rows: the weights are read once per launch for all the tokens.
//
// Work comes in items of 128 weight rows x one chunk of K (small_ck<NT>()
// elements, whole 256-element blocks: 512 up to 16 tokens, 256 above, so that
// the stages fit in shared memory).  Where the epilogue allows it (not
// SwiGLU, which needs whole sums) every chunk of K is an independent item
// whose partial rows are added to y with atomics; for SwiGLU a CTA runs the
// chunks of a row tile in order and stores the whole sums.  The grid is
// persistent (the resident CTAs) and takes items in turn through a ring of
// cp.async stages: everything an item reads -- the rows' packed codes,
// sub-block scales, split minima, block scales and min shifts, the
// activations' exact hi / lo FP16 split and their sub-block sums -- is copied
// into its stage while earlier items compute, so a CTA waits on memory once
// per launch rather than once per chunk.  The weights do not depend on the
// previous kernel: the first item's are requested before the programmatic
// launch wait, its activations after it.
//
// Compute (per warp: 16 rows; per lane: rows gq and gq + 8): per 32-element
// sub-block a lane takes one 32-bit word of each of its two rows (bytes
// 4tq .. 4tq + 3 of the row's 16 packed bytes: elements 4tq .. 4tq + 3 in the
// low nibbles, 16 + 4tq .. in the high ones) and builds the A fragments of
// both K-halves from it, sc*q exact in FP16 as in tc_gemm_q4kp_kernel.  The
// fragment's K order is a fixed permutation of the sub-block's (logical k
// 2tq + e <-> element 4tq + e, 2tq + 8 + e <-> element 4tq + 2 + e); the
// activations are read with the same permutation, so every dot product is
// unchanged.  Each group of four sub-blocks accumulates on its own (in four
// independent chains up to 16 tokens) and is added with its block's scale d.  The min term sum_sub dmin*m * sum(x) is
// four more MMAs per item: the rows' exact hi / lo FP16 split of
// dmin*m*2^shift against the tokens' hi / lo sub-block sums, K = the item's
// sub-blocks.  Up to 16 tokens a CTA runs two warp groups, each on half of
// an item's sub-blocks (the register budget allows it there), and the groups'
// sums meet in shared memory before the output.
constexpr int kSmallRows = 128;
constexpr int kSmallThreads = 256;

__device__ __forceinline__ void mma_16816(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// cp.async of 16 / 8 / 4 bytes; `valid` bytes are read from src (0: the
// destination is zero-filled and src is not read).
__device__ __forceinline__ void cpa16(void* dst, const void* src, unsigned valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid)
                 : "memory");
}
__device__ __forceinline__ void cpa8(void* dst, const void* src, unsigned valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid)
                 : "memory");
}
__device__ __forceinline__ void cpa4(void* dst, const void* src, unsigned valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid)
                 : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int NT>
constexpr int small_ck() { return NT <= 2 ? 512 : 256; }

// One stage of the small-batch ring: byte offsets of its arrays.
template <int NT>
struct SmallStage {
    static constexpr int CK = small_ck<NT>(), CU = CK / 32, CB = CK / 256, MT = 8 * NT;
    static constexpr int WS = CU * 16 + 16;  // a row's codes, padded: conflict-free fragment loads
    static constexpr int XS = CK * 2 + 32;   // a token's hi (or lo) activations, padded likewise
    static constexpr int kCodes = 0;                                  // [rows][WS]
    static constexpr int kX = kCodes + kSmallRows * WS;               // hi, then lo: [MT][XS] each
    static constexpr int kSum = kX + 2 * MT * XS;                     // shi, then slo: [MT][CU] halves each
    static constexpr int kMin = kSum + 2 * MT * CU * 2;               // qmin hi, then lo: [rows][CU] halves each
    static constexpr int kSc = kMin + 2 * kSmallRows * CU * 2;        // [rows][CU] bytes
    static constexpr int kD = kSc + kSmallRows * CU;                  // [rows][CB] floats
    static constexpr int kShift = kD + kSmallRows * CB * 4;           // [rows] min shifts
    static constexpr int kBytes = (kShift + kSmallRows + 127) / 128 * 128;
    // as many stages (2..3) as fit beside one another in 220 KB
    static constexpr int kStages = 3 * kBytes <= 220 * 1024 ? 3 : 2;
};
template <int NT>
constexpr int small_groups() { return NT <= 2 ? 2 : 1; }  // warp groups of eight per CTA
// the stages, then (two groups) the second group's partial sums [rows][MT]
template <int NT>
constexpr std::size_t small_smem_bytes() {
    return std::size_t(SmallStage<NT>::kStages) * SmallStage<NT>::kBytes +
           (small_groups<NT>() > 1 ? std::size_t(kSmallRows) * 8 * NT * 4 : 0);
}
constexpr int small_log2(int v) { return v <= 1 ? 0 : 1 + small_log2(v / 2); }

struct SmallWork {
    int row_tiles;    // 128-row tiles
    int pairs;        // row tiles x K slices
    int slice_units;  // sub-blocks per K slice (whole blocks)
    int chunks;       // items per (row tile, slice)
};

template <int NT>  // 8-token tiles: up to 8 * NT tokens
__global__ void __launch_bounds__(kSmallThreads * small_groups<NT>(), 1) gemm_small_q4k_kernel(DeviceMatrix w, const __half* xhi,
                                                                         const __half* xlo, const int* xshift,
                                                                         const __half* shi, const __half* slo,
                                                                         int tokens, SmallWork wk, float* y, int ldy,
                                                                         int epilogue, int atomic) {
    using S = SmallStage<NT>;
    constexpr int MT = S::MT, CU = S::CU, CB = S::CB, WS = S::WS, XS = S::XS, NS = S::kStages;
    constexpr int G = small_groups<NT>(), TH = kSmallThreads * G, LMT = small_log2(MT);
    extern __shared__ __align__(128) unsigned char small_smem[];
    const int units = w.cols / 32, kblocks = w.cols / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int mine = wk.pairs > int(blockIdx.x) ? (wk.pairs - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
    const int n_items = mine * wk.chunks;

    // Items in the order this CTA takes them: its (row tile, slice) pairs
    // blockIdx.x, + gridDim.x, ..., each as `chunks` consecutive chunks.  A
    // cursor walks them without divisions; one runs ahead for the copies.
    struct Cursor {
        int rt, sp, c;
        __device__ void next(const SmallWork& wk) {
            if (++c < wk.chunks) return;
            c = 0;
            rt += int(gridDim.x);
            while (rt >= wk.row_tiles) {
                rt -= wk.row_tiles;
                ++sp;
            }
        }
    };
    struct Item {
        int row0, u_begin, cu;
        bool first, last;
    };
    auto item = [&](const Cursor& k) {
        const int lo = k.sp * wk.slice_units, hi = min(lo + wk.slice_units, units);
        Item it;
        it.row0 = k.rt * kSmallRows;
        it.u_begin = lo + k.c * CU;
        it.cu = min(CU, hi - it.u_begin);  // 8 or 16 (whole blocks)
        it.first = k.c == 0;
        it.last = k.c == wk.chunks - 1;
        return it;
    };
    // the weight-side copies of an item into stage st: each thread keeps one
    // 16-byte column of the rows and steps down them
    auto issue_weights = [&](const Item& it, int st) {
        unsigned char* b = small_smem + st * S::kBytes;
        {
            const int lg = it.cu == 16 ? 4 : 3, k = threadIdx.x & (it.cu - 1), rp = TH >> lg;
            int r = threadIdx.x >> lg;
            const unsigned char* src = w.qs + (long long)(it.row0 + r) * (long long)w.qs_row + (it.u_begin + k) * 16;
            unsigned char* dst = b + S::kCodes + r * WS + k * 16;
            const long long step = (long long)rp * (long long)w.qs_row;
            for (; r < kSmallRows; r += rp, src += step, dst += rp * WS) {
                const bool ok = it.row0 + r < w.rows;
                cpa16(dst, ok ? src : w.qs, ok ? 16u : 0u);
            }
        }
        {
            const int c8 = it.cu >> 3, k = threadIdx.x & (c8 - 1), r = threadIdx.x >> (c8 - 1);
            if (r < kSmallRows) {  // TH / c8 >= 128: one piece per array and thread at most
                const int row = it.row0 + r;
                const bool ok = row < w.rows;
                const long long off = (long long)(ok ? row : 0) * units + it.u_begin + 8 * k;
                cpa8(b + S::kSc + r * CU + 8 * k, w.qsc + off, ok ? 8u : 0u);
                cpa16(b + S::kMin + (r * CU + 8 * k) * 2, w.qmin_hi + off, ok ? 16u : 0u);
                cpa16(b + S::kMin + (kSmallRows * CU + r * CU + 8 * k) * 2, w.qmin_lo + off, ok ? 16u : 0u);
                cpa4(b + S::kD + (r * CB + k) * 4,
                     w.qscale + (long long)(ok ? row : 0) * kblocks + it.u_begin / 8 + k, ok ? 4u : 0u);
            }
        }
        if (threadIdx.x < kSmallRows / 4) {
            const int r = 4 * threadIdx.x;
            const int have = max(0, min(4, w.rows - (it.row0 + r)));
            cpa4(b + S::kShift + r, w.qmin_shift + (have ? it.row0 + r : 0), unsigned(have));
        }
    };
    // the activation-side copies of an item into stage st (rows: hi tokens, then lo)
    auto issue_acts = [&](const Item& it, int st) {
        unsigned char* b = small_smem + st * S::kBytes;
        {
            const int lp = it.cu == 16 ? 6 : 5;  // 16-byte pieces per token row: cu * 4
            const int k = threadIdx.x & ((1 << lp) - 1), rp = TH >> lp;
            for (int q = threadIdx.x >> lp; q < 2 * MT; q += rp) {
                const int part = q >> LMT, t = q & (MT - 1);
                const bool ok = t < tokens;
                const __half* src = (part ? xlo : xhi) + (long long)(ok ? t : 0) * w.cols + it.u_begin * 32 + 8 * k;
                cpa16(b + S::kX + q * XS + 16 * k, src, ok ? 16u : 0u);
            }
        }
        {
            const int c8 = it.cu >> 3, k = threadIdx.x & (c8 - 1), q = threadIdx.x >> (c8 - 1);
            if (q < 2 * MT) {
                const int part = q >> LMT, t = q & (MT - 1);
                const bool ok = t < tokens;
                const __half* src = (part ? slo : shi) + (long long)(ok ? t : 0) * units + it.u_begin + 8 * k;
                cpa16(b + S::kSum + (q * CU + 8 * k) * 2, src, ok ? 16u : 0u);
            }
        }
    };

    // prologue: item 0's weights before the wait on the previous kernel, its
    // activations after it; then the rest of the ring
    Cursor ic{int(blockIdx.x) % wk.row_tiles, int(blockIdx.x) / wk.row_tiles, 0};
    Cursor cc = ic;
    int issued = 0;
    if (issued < n_items) issue_weights(item(ic), 0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (issued < n_items) {
        issue_acts(item(ic), 0);
        ic.next(wk);
        ++issued;
    }
    cpa_commit();
#pragma unroll
    for (int s = 1; s < NS - 1; ++s) {
        if (issued < n_items) {
            const Item it = item(ic);
            issue_weights(it, s);
            issue_acts(it, s);
            ic.next(wk);
            ++issued;
        }
        cpa_commit();
    }
    float xs[NT][2];  // 2^-shift of the lane's output tokens
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int t = 8 * n + 2 * tq + e;
            xs[n][e] = t < tokens ? pow2(-__ldg(xshift + t)) : 0.f;
        }

    const int wg = warp >> 3;                           // warp group
    const int la = (warp & 7) * 16 + gq, lb = la + 8;  // the lane's rows within the tile
    float* red = reinterpret_cast<float*>(small_smem + NS * S::kBytes);  // [rows][MT] (two groups)
    float tot[NT][4];
    for (int j = 0; j < n_items; ++j) {
        cpa_wait<NS - 2>();
        __syncthreads();  // item j's stage is complete; the stage refilled below is no longer read
        if (issued < n_items) {  // item j + NS - 1
            const Item nx = item(ic);
            issue_weights(nx, (j + NS - 1) % NS);
            issue_acts(nx, (j + NS - 1) % NS);
            ic.next(wk);
            ++issued;
        }
        cpa_commit();

        const Item it = item(cc);
        cc.next(wk);
        const unsigned char* b = small_smem + (j % NS) * S::kBytes;
        const unsigned char* codes = b + S::kCodes;
        const unsigned char* xh_s = b + S::kX;
        const unsigned char* xl_s = b + S::kX + MT * XS;
        if (it.first) {
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) tot[n][e] = 0.f;
        }
        const int half = it.cu / G;  // this group's sub-blocks: [wg * half, (wg + 1) * half)
        for (int u4 = wg * half; u4 < (wg + 1) * half; u4 += 4) {
            const int bk = u4 >> 3;  // the sub-blocks' 256-element block
            const float da = reinterpret_cast<const float*>(b + S::kD)[la * CB + bk];
            const float db = reinterpret_cast<const float*>(b + S::kD)[lb * CB + bk];
            const unsigned ga = *reinterpret_cast<const unsigned*>(b + S::kSc + la * CU + u4);
            const unsigned gbk = *reinterpret_cast<const unsigned*>(b + S::kSc + lb * CU + u4);
            // NA independent accumulator chains per token tile (hi / lo part x
            // sub-block parity) when there are too few tiles to hide the MMA latency
            constexpr int NA = NT <= 2 ? 4 : 1;
            float blk[NA][NT][4];
#pragma unroll
            for (int c = 0; c < NA; ++c)
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) blk[c][n][e] = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int u = u4 + i;  // sub-block within the item
                const unsigned wa = *reinterpret_cast<const unsigned*>(codes + la * WS + u * 16 + 4 * tq);
                const unsigned wb = *reinterpret_cast<const unsigned*>(codes + lb * WS + u * 16 + 4 * tq);
                // sc (below 64) in both halves: 0x64xx = 1024 + sc exactly, minus 1024
                const __half2 k1024 = __half2half2(__ushort_as_half(0x6400)), km1024 = __hneg2(k1024);
                const unsigned qa = __byte_perm(ga, 0x64646464u, 0x4040u + 0x0101u * i);
                const unsigned qb = __byte_perm(gbk, 0x64646464u, 0x4040u + 0x0101u * i);
                const __half2 sa2 = __hsub2(*reinterpret_cast<const __half2*>(&qa), k1024);
                const __half2 sb2 = __hsub2(*reinterpret_cast<const __half2*>(&qb), k1024);
                const __half2 oa2 = __hmul2(sa2, km1024), ob2 = __hmul2(sb2, km1024);
#pragma unroll
                for (int hk = 0; hk < 2; ++hk) {  // low nibbles: elements 0..15, high: 16..31
                    const unsigned ma = hk ? (wa >> 4) & 0x0F0F0F0Fu : wa & 0x0F0F0F0Fu;
                    const unsigned mb = hk ? (wb >> 4) & 0x0F0F0F0Fu : wb & 0x0F0F0F0Fu;
                    unsigned a[4];
                    const unsigned p0 = __byte_perm(ma, 0x64646464u, 0x4140), p1 = __byte_perm(mb, 0x64646464u, 0x4140);
                    const unsigned p2 = __byte_perm(ma, 0x64646464u, 0x4342), p3 = __byte_perm(mb, 0x64646464u, 0x4342);
                    const __half2 h0 = __hfma2(*reinterpret_cast<const __half2*>(&p0), sa2, oa2);
                    const __half2 h1 = __hfma2(*reinterpret_cast<const __half2*>(&p1), sb2, ob2);
                    const __half2 h2 = __hfma2(*reinterpret_cast<const __half2*>(&p2), sa2, oa2);
                    const __half2 h3 = __hfma2(*reinterpret_cast<const __half2*>(&p3), sb2, ob2);
                    a[0] = *reinterpret_cast<const unsigned*>(&h0);  // row gq, elements 4tq, 4tq + 1
                    a[1] = *reinterpret_cast<const unsigned*>(&h1);  // row gq + 8
                    a[2] = *reinterpret_cast<const unsigned*>(&h2);  // row gq, elements 4tq + 2, 4tq + 3
                    a[3] = *reinterpret_cast<const unsigned*>(&h3);
                    const int koff = (u * 32 + 16 * hk + 4 * tq) * 2;
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const uint2 bh = *reinterpret_cast<const uint2*>(xh_s + (8 * n + gq) * XS + koff);
                        const uint2 bl = *reinterpret_cast<const uint2*>(xl_s + (8 * n + gq) * XS + koff);
                        mma_16816(blk[NA > 1 ? 2 * (i & 1) : 0][n], a, bh.x, bh.y);
                        mma_16816(blk[NA > 1 ? 2 * (i & 1) + 1 : 0][n], a, bl.x, bl.y);
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = blk[0][n][e];
#pragma unroll
                    for (int c = 1; c < NA; ++c) v += blk[c][n][e];
                    tot[n][e] = fmaf(e < 2 ? da : db, v, tot[n][e]);
                }
        }
        if (wg == 0) {
            // min term: - 2^-shift * 32 * sum_sub (hi + lo)(dmin*m*2^shift) * (hi + lo)(sum x * 2^(xshift - 5)),
            // one m16n8k16 per pair of parts with K = the item's sub-blocks (the upper eight are zero
            // when the item has eight)
            const signed char* shf = reinterpret_cast<const signed char*>(b + S::kShift);
            const float fa = pow2(-shf[la]) * 32.f, fb = pow2(-shf[lb]) * 32.f;
            const unsigned char* mhi = b + S::kMin;
            const unsigned char* mlo = mhi + kSmallRows * CU * 2;
            const unsigned char* sh = b + S::kSum;
            const unsigned char* sl = sh + MT * CU * 2;
            const bool upper = CU == 16 && it.cu == 16;
            auto word = [&](const unsigned char* base, int r, int u, bool ok) {
                return ok ? *reinterpret_cast<const unsigned*>(base + (r * CU + u) * 2) : 0u;
            };
            const unsigned ah[4] = {word(mhi, la, 2 * tq, true), word(mhi, lb, 2 * tq, true),
                                    word(mhi, la, 2 * tq + 8, upper), word(mhi, lb, 2 * tq + 8, upper)};
            const unsigned al[4] = {word(mlo, la, 2 * tq, true), word(mlo, lb, 2 * tq, true),
                                    word(mlo, la, 2 * tq + 8, upper), word(mlo, lb, 2 * tq + 8, upper)};
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int t = 8 * n + gq;
                const unsigned bh0 = word(sh, t, 2 * tq, true), bh1 = word(sh, t, 2 * tq + 8, upper);
                const unsigned bl0 = word(sl, t, 2 * tq, true), bl1 = word(sl, t, 2 * tq + 8, upper);
                float m[4] = {0.f, 0.f, 0.f, 0.f};
                mma_16816(m, ah, bh0, bh1);
                mma_16816(m, ah, bl0, bl1);
                mma_16816(m, al, bh0, bh1);
                mma_16816(m, al, bl0, bl1);
                tot[n][0] = fmaf(-fa, m[0], tot[n][0]);
                tot[n][1] = fmaf(-fa, m[1], tot[n][1]);
                tot[n][2] = fmaf(-fb, m[2], tot[n][2]);
                tot[n][3] = fmaf(-fb, m[3], tot[n][3]);
            }
        }
        if (!it.last) continue;
        if (G > 1) {  // the second group's sums join the first's
            if (wg == 1) {
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        red[(e < 2 ? la : lb) * MT + 8 * n + 2 * tq + (e & 1)] = tot[n][e];
            }
            __syncthreads();
            if (wg == 1) continue;
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) tot[n][e] += red[(e < 2 ? la : lb) * MT + 8 * n + 2 * tq + (e & 1)];
        }
        // out: accumulator (row gq / gq + 8, tokens 8n + 2tq, + 1), scaled back by 2^-shift
        const int row_a = it.row0 + la, row_b = it.row0 + lb;
        const bool live_a = row_a < w.rows, live_b = row_b < w.rows;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = 8 * n + 2 * tq + (e & 1);
                const bool rlive = e < 2 ? live_a : live_b;
                const int row = e < 2 ? row_a : row_b;
                const float v = tot[n][e] * xs[n][e & 1];
                if (epilogue == kSwiGLU) {
                    // rows (2i, 2i + 1) = (gate_i, up_i) sit in lanes gq and gq ^ 1 (4 lanes apart)
                    const float other = __shfl_xor_sync(0xffffffffu, v, 4);
                    if (rlive && t < tokens && !(gq & 1)) y[(long long)t * ldy + row / 2] = swiglu_12(v, other);
                } else if (rlive && t < tokens) {
                    float* dst = y + (long long)t * ldy + row;
                    if (atomic || epilogue == kAdd) atomicAdd(dst, v);
                    else *dst = v;
                }
            }
    }
    cpa_wait<0>();  // no copy is left in flight when the CTA exits
}

// ---------------------------------------------------------------------------
// Small batches (5 .. 32 tokens) of Q8_0 / Q4_0 rows on mma.sync, straight
// from the packed rows, with the activations' exact hi / lo FP16 split of
// split_kernel.  A Q8_0 code is an int8, a Q4_0 code minus 8 lies in -8..7:
// both are exact in FP16 (a byte permute onto 0x64xx = 1024 + byte and one
// half2 subtraction), so each 32-element block's products are exact and its
// two k16 MMAs (hi and lo chains) accumulate in F32 before the block is added
// with its scale d.  A CTA is eight warps on 128 weight rows (16 per warp),
// one slice of K and up to 32 tokens.  Per
// block a lane takes, of each of its two rows, the 8 code bytes 8tq .. 8tq+7
// (Q8_0, one 8-byte load) or the code word tq (Q4_0: elements 4tq .. 4tq+3
// in the low nibbles, 16 + 4tq .. in the high ones), from a register ring
// kSmallQDepth blocks ahead, with the block's fp16 scale d.  The fragments' K order is a fixed
// permutation of the block's (Q8_0: k16 #0 <- elements {0-3, 8-11, 16-19,
// 24-27}, #1 <- the rest; Q4_0: #0 <- the low nibbles, #1 <- the high ones),
// and the activations are read with the same permutation, so every dot
// product is unchanged.  Shared-memory rows of x are padded so that the
// fragment loads are free of bank conflicts.
constexpr int kSmallQChunk = 256;  // K elements of x staged at a time: 8 blocks
constexpr int kSmallQDepth = 8;    // blocks of packed codes in flight per lane
constexpr int kSmallQMaxTokens = 32;  // above it the exact-plane kernels are faster

template <int TYPE>
constexpr int smallq_xs() { return kSmallQChunk * 2 + (TYPE == kQ8_0 ? 64 : 32); }  // bytes per token row
template <int TYPE>
constexpr std::size_t smallq_smem_bytes(int nt) { return std::size_t(8 * nt) * smallq_xs<TYPE>() * 2; }

__device__ __forceinline__ void mma_16816_z(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Two FP16 codes (bytes sel of w, w already biased to 0..255) as a half2 minus bias.
__device__ __forceinline__ unsigned code_pair(unsigned w, unsigned sel, __half2 bias) {
    const unsigned p = __byte_perm(w, 0x64646464u, sel);
    const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&p), bias);
    return *reinterpret_cast<const unsigned*>(&h);
}

template <int TYPE, int NT>  // 8-token tiles: up to 8 * NT tokens per CTA
__global__ void __launch_bounds__(kSmallThreads) gemm_small_q8_kernel(DeviceMatrix w, const __half* xhi,
                                                                     const __half* xlo, const int* xshift, int tokens,
                                                                     int kslice, float* y, int ldy, int epilogue,
                                                                     int atomic) {
    static_assert(TYPE == kQ8_0 || TYPE == kQ4_0, "Q8_0 / Q4_0 only");
    constexpr int MT = 8 * NT;
    constexpr int XS = smallq_xs<TYPE>();
    constexpr int CB = kSmallQChunk / 32;  // blocks per chunk
    static_assert(CB == kSmallQDepth, "the ring holds one chunk of blocks");
    using Word = std::conditional_t<TYPE == kQ8_0, uint2, unsigned>;
    constexpr int kBlockBytes = TYPE == kQ8_0 ? 32 : 16;  // packed code bytes per block
    extern __shared__ __align__(16) unsigned char smallq_smem[];
    unsigned char* xh_s = smallq_smem;
    unsigned char* xl_s = xh_s + MT * XS;
    const int t0 = blockIdx.z * MT;             // first token of this CTA
    const int b0 = blockIdx.y * (kslice / 32);  // first block of this CTA's slice
    const int sb = kslice / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int row_a = blockIdx.x * kSmallRows + warp * 16 + gq, row_b = row_a + 8;
    const bool live_a = row_a < w.rows, live_b = row_b < w.rows;
    const long long ra = live_a ? row_a : 0, rb = live_b ? row_b : 0;
    const unsigned char* qa = w.qs + ra * (long long)w.qs_row + (long long)b0 * kBlockBytes +
                              (TYPE == kQ8_0 ? 8 * tq : 4 * tq);
    const unsigned char* qb = w.qs + rb * (long long)w.qs_row + (long long)b0 * kBlockBytes +
                              (TYPE == kQ8_0 ? 8 * tq : 4 * tq);
    const unsigned short* da_p = reinterpret_cast<const unsigned short*>(w.meta + ra * (long long)w.meta_row) + b0;
    const unsigned short* db_p = reinterpret_cast<const unsigned short*>(w.meta + rb * (long long)w.meta_row) + b0;
    auto load = [&](const unsigned char* q, int i) -> Word {
        return *reinterpret_cast<const Word*>(q + (long long)i * kBlockBytes);
    };
    float tot[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) tot[n][e] = 0.f;
    Word ring_a[kSmallQDepth], ring_b[kSmallQDepth];
    unsigned short dr_a[kSmallQDepth], dr_b[kSmallQDepth];
#pragma unroll
    for (int i = 0; i < kSmallQDepth; ++i) {
        ring_a[i] = i < sb ? load(qa, i) : Word{};
        ring_b[i] = i < sb ? load(qb, i) : Word{};
        dr_a[i] = i < sb ? da_p[i] : 0;
        dr_b[i] = i < sb ? db_p[i] : 0;
    }
    const __half2 bias = __half2half2(__ushort_as_half(TYPE == kQ8_0 ? 0x6480 : 0x6408));  // 1152 / 1032
    for (int c0 = 0; c0 < sb; c0 += CB) {
        const int cb = min(CB, sb - c0);
        __syncthreads();  // the previous chunk of x is no longer read
        for (int i = threadIdx.x; i < MT * cb * 4; i += blockDim.x) {
            const int t = i / (cb * 4), c = i % (cb * 4);  // c: 8 elements (16 bytes)
            uint4 h = make_uint4(0, 0, 0, 0), l = h;
            if (t0 + t < tokens) {
                const long long off = (long long)(t0 + t) * w.cols + (long long)(b0 + c0) * 32 + 8 * c;
                h = *reinterpret_cast<const uint4*>(xhi + off);
                l = *reinterpret_cast<const uint4*>(xlo + off);
            }
            *reinterpret_cast<uint4*>(xh_s + t * XS + 16 * c) = h;
            *reinterpret_cast<uint4*>(xl_s + t * XS + 16 * c) = l;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kSmallQDepth; ++i) {
            if (i >= cb) break;  // uniform: a short last chunk
            const Word wa = ring_a[i], wb = ring_b[i];
            const float da = live_a ? __half2float(__ushort_as_half(dr_a[i])) : 0.f;
            const float db = live_b ? __half2float(__ushort_as_half(dr_b[i])) : 0.f;
            const int nxt = c0 + i + kSmallQDepth;
            if (nxt < sb) {
                ring_a[i] = load(qa, nxt);
                ring_b[i] = load(qb, nxt);
                dr_a[i] = da_p[nxt];
                dr_b[i] = db_p[nxt];
            }
            unsigned A0[4], A1[4];
            if constexpr (TYPE == kQ8_0) {
                const unsigned ax = wa.x ^ 0x80808080u, ay = wa.y ^ 0x80808080u;
                const unsigned bx = wb.x ^ 0x80808080u, by = wb.y ^ 0x80808080u;
                A0[0] = code_pair(ax, 0x4140, bias);
                A0[1] = code_pair(bx, 0x4140, bias);
                A0[2] = code_pair(ax, 0x4342, bias);
                A0[3] = code_pair(bx, 0x4342, bias);
                A1[0] = code_pair(ay, 0x4140, bias);
                A1[1] = code_pair(by, 0x4140, bias);
                A1[2] = code_pair(ay, 0x4342, bias);
                A1[3] = code_pair(by, 0x4342, bias);
            } else {
                const unsigned al = wa & 0x0F0F0F0Fu, ah = (wa >> 4) & 0x0F0F0F0Fu;
                const unsigned bl = wb & 0x0F0F0F0Fu, bh = (wb >> 4) & 0x0F0F0F0Fu;
                A0[0] = code_pair(al, 0x4140, bias);
                A0[1] = code_pair(bl, 0x4140, bias);
                A0[2] = code_pair(al, 0x4342, bias);
                A0[3] = code_pair(bl, 0x4342, bias);
                A1[0] = code_pair(ah, 0x4140, bias);
                A1[1] = code_pair(bh, 0x4140, bias);
                A1[2] = code_pair(ah, 0x4342, bias);
                A1[3] = code_pair(bh, 0x4342, bias);
            }
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int xo = (8 * n + gq) * XS;
                unsigned h[4], l[4];  // B of k16 #0 (h[0], h[1]) and #1 (h[2], h[3])
                if constexpr (TYPE == kQ8_0) {
                    const int ko = (i * 32 + 8 * tq) * 2;  // elements 8tq .. 8tq + 7
                    const uint4 vh = *reinterpret_cast<const uint4*>(xh_s + xo + ko);
                    const uint4 vl = *reinterpret_cast<const uint4*>(xl_s + xo + ko);
                    h[0] = vh.x, h[1] = vh.y, h[2] = vh.z, h[3] = vh.w;
                    l[0] = vl.x, l[1] = vl.y, l[2] = vl.z, l[3] = vl.w;
                } else {
                    const int k0 = (i * 32 + 4 * tq) * 2, k1 = k0 + 32;  // elements 4tq .., 16 + 4tq ..
                    const uint2 h0 = *reinterpret_cast<const uint2*>(xh_s + xo + k0);
                    const uint2 h1 = *reinterpret_cast<const uint2*>(xh_s + xo + k1);
                    const uint2 l0 = *reinterpret_cast<const uint2*>(xl_s + xo + k0);
                    const uint2 l1 = *reinterpret_cast<const uint2*>(xl_s + xo + k1);
                    h[0] = h0.x, h[1] = h0.y, h[2] = h1.x, h[3] = h1.y;
                    l[0] = l0.x, l[1] = l0.y, l[2] = l1.x, l[3] = l1.y;
                }
                float ch[4], cl[4];
                mma_16816_z(ch, A0, h[0], h[1]);
                mma_16816_z(cl, A0, l[0], l[1]);
                mma_16816(ch, A1, h[2], h[3]);
                mma_16816(cl, A1, l[2], l[3]);
                tot[n][0] = fmaf(da, ch[0] + cl[0], tot[n][0]);
                tot[n][1] = fmaf(da, ch[1] + cl[1], tot[n][1]);
                tot[n][2] = fmaf(db, ch[2] + cl[2], tot[n][2]);
                tot[n][3] = fmaf(db, ch[3] + cl[3], tot[n][3]);
            }
        }
    }
    // out: accumulator (row gq / gq + 8, tokens t0 + 8n + 2tq, + 1), scaled back by 2^-shift
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = t0 + 8 * n + 2 * tq + (e & 1);
            const bool rlive = e < 2 ? live_a : live_b;
            const int row = e < 2 ? row_a : row_b;
            const float v = t < tokens ? tot[n][e] * pow2(-xshift[t]) : 0.f;
            if (epilogue == kSwiGLU) {
                // rows (2i, 2i + 1) = (gate_i, up_i) sit in lanes gq and gq ^ 1 (4 lanes apart)
                const float other = __shfl_xor_sync(0xffffffffu, v, 4);
                if (rlive && t < tokens && !(gq & 1)) y[(long long)t * ldy + row / 2] = swiglu_12(v, other);
            } else if (rlive && t < tokens) {
                float* dst = y + (long long)t * ldy + row;
                if (atomic || epilogue == kAdd) atomicAdd(dst, v);
                else *dst = v;
            }
        }
}

// X [T][K] F32 -> hi, lo FP16 [T][K] with a per-token power-of-two scale
// that puts max|x| in [2^14, 2^15), then the exact split (split.cuh).  One
// block per token; float4 loads and 8-byte stores (K % 4 == 0, rows 16-byte
// aligned, which the launcher checks).
__global__ void split_kernel(const float* x, int ldx, int K, __half* hi, __half* lo, int* shift, __half* shi,
                             __half* slo) {
    // a programmatically launched projection may start its weight copies now;
    // it reads these outputs only after its grid-dependency wait
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int t = blockIdx.x;
    const float4* row = reinterpret_cast<const float4*>(x + (long long)t * ldx);
    const int K4 = K / 4;
    float m = 0.f;
    for (int k = threadIdx.x; k < K4; k += blockDim.x) {
        const float4 v = row[k];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    __shared__ float sm[32];
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) sm[0] = v;
    }
    __syncthreads();
    int e = 0;
    if (sm[0] > 0.f && isfinite(sm[0])) frexpf(sm[0], &e);
    const int s = sm[0] > 0.f ? max(-100, min(100, 15 - e)) : 0;
    if (threadIdx.x == 0) shift[t] = s;
    const float f = pow2(s);
    uint2* hrow = reinterpret_cast<uint2*>(hi + (long long)t * K);
    uint2* lrow = reinterpret_cast<uint2*>(lo + (long long)t * K);
    const bool sums = K % 32 == 0;  // the Q4_K min term's sub-block sums
    const float f32 = pow2(s - 5);
    for (int k0 = 0; k0 < K4; k0 += blockDim.x) {  // uniform trip count (shuffles)
        const int k = k0 + threadIdx.x;
        const float4 v = k < K4 ? row[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < K4) {
            uint2 h, l;
            split_exact(v.x * f, v.y * f, h.x, l.x);
            split_exact(v.z * f, v.w * f, h.y, l.y);
            hrow[k] = h;
            lrow[k] = l;
        }
        if (sums) subblock_sum_split(v, k, k < K4, f32, shi + (long long)t * (K / 32), slo + (long long)t * (K / 32));
    }
}

// ---------------------------------------------------------------- host side
CUtensorMap make_map(const __half* base, int K, int T, int n_tile) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(T)};
    const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(n_tile)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides,
                                   box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

// Packed Q4_K rows as a 2-D byte tensor: the 16 bytes of one sub-block of
// each of a tile's 128 rows per box (no swizzle: producers read row r at r*16).
// steps > 1: a box of `steps` sub-blocks (16 * steps bytes) per row, with the
// 64-byte swizzle (producers read step i of row r at sw64(r, i)).
CUtensorMap make_packed_map(const std::uint8_t* qs, std::size_t row_bytes, int rows, int steps = 1) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(row_bytes), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
    const cuuint32_t box[2] = {cuuint32_t(16 * steps), cuuint32_t(kBM)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<std::uint8_t*>(qs), dims,
                                            strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            steps > 1 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

template <int TYPE>
void run_tc(const CUtensorMap& hi, const CUtensorMap& lo, const CUtensorMap& ahi, const CUtensorMap& alo,
            const TcArgs& a, dim3 grid, cudaStream_t s) {
    const int smem = kStages * (2 * kATile + 2 * kBTileMax) + 1024 + 256;
    // a per-device attribute: set on every launch (about a microsecond)
    TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    tc_gemm_kernel<TYPE><<<grid, kThreads, smem, s>>>(hi, lo, ahi, alo, a);
    TVARA_LAUNCHED();
}

int g_tc_min_tokens = 5;  // below this the CUDA-core GEMV streams weights once per <=4 tokens
bool g_small_batches = true;  // 5..64 tokens of packed Q4_K rows: gemm_small_q4k_kernel
bool g_tc_persistent = true;  // plane path: persistent kernel (else one CTA per tile)

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return n > 0 ? n : 148;
}

struct TilePlan {
    int n_tile, token_tiles, splits;
};

// Token tile width and split-K count for a launch: one CTA per SM, so the
// time is about (waves) x (per-tile time), and a partial last wave costs a
// whole one.  Candidates: balanced token tiles (width a multiple of 16, at
// most 256) and power-of-two K splits of at least 8 steps (none for SwiGLU,
// which is nonlinear).  Per tile: K-steps x (width + a fixed per-step cost)
// plus a fixed cost for the pipeline fill and the epilogue (which grows with
// the width and, for split K, with the atomic accumulation).
// flat_step > 0 (the tensor-memory Q4_K forms): a K-step costs about the
// same at any tile width up to the maximum (the pace is set by the x-tile
// round trip, not the MMA width: measured ~600 cycles at widths 96..192), so
// wide tiles with split K beat narrow unsplit ones; the pipeline fill (two
// stages) is charged per tile.  whole_blocks: splits divide the 256-element
// blocks (8 K-steps).
TilePlan plan_tiles(int row_tiles, int tokens, int steps, bool can_split, int sms, int max_n = kMaxN,
                    double flat_step = 0.0, bool whole_blocks = false) {
    TilePlan best{0, 0, 0};
    double best_cost = 0;
    for (int tt = (tokens + max_n - 1) / max_n; tt <= (tokens + 15) / 16 && tt <= 64; ++tt) {
        const int width = (((tokens + tt - 1) / tt) + 15) / 16 * 16;
        if (width > max_n) continue;
        const int token_tiles = (tokens + width - 1) / width;
        for (int sp = 1; sp <= 16; sp *= 2) {
            if (sp > 1 && (!can_split || steps % sp || steps / sp < 8)) break;
            if (sp > 1 && whole_blocks && (steps / 8) % sp) continue;
            const long long tiles = (long long)row_tiles * token_tiles * sp;
            const long long waves = (tiles + sms - 1) / sms;
            const double step_cost = flat_step > 0 ? flat_step : double(width + 48);
            const double per_tile = double(steps / sp) * step_cost + (flat_step > 0 ? 8.0 * flat_step : 0.0) + 6.0 * width +
                                    1500.0 + (sp > 1 ? 8.0 * width : 0.0);
            const double cost = double(waves) * per_tile;
            if (!best.n_tile || cost < best_cost) {
                best = {width, token_tiles, sp};
                best_cost = cost;
            }
        }
    }
    return best;
}

}  // namespace

bool gemm_tc_supported(const DeviceMatrix& w, int tokens) {
    return tokens >= g_tc_min_tokens && w.cols % kBK == 0 && w.row_shift != nullptr;
}

std::size_t gemm_tc_workspace(int max_tokens, int max_cols) {
    // hi + lo activations, per-token shifts (padded to 64), an error flag,
    // hi + lo sub-block sums (the Q4_K min term)
    return std::size_t(max_tokens) * max_cols * 2 * sizeof(__half) +
           std::size_t((max_tokens + 63) / 64 * 64 + 64) * sizeof(int) +
           std::size_t(max_tokens) * (max_cols / 32) * 2 * sizeof(__half) + 2048;
}

void gemm_tc_split_buffers(void* workspace, std::size_t workspace_bytes, int tokens, int cols, __half*& hi,
                           __half*& lo, int*& shift, __half** shi, __half** slo) {
    if (!workspace || workspace_bytes < gemm_tc_workspace(tokens, cols))
        throw std::invalid_argument("tensor-core projection workspace too small");
    hi = static_cast<__half*>(workspace);
    lo = hi + std::size_t(tokens) * cols;
    shift = reinterpret_cast<int*>(lo + std::size_t(tokens) * cols);
    // after the shifts and the workspace's error slot
    auto* s0 = reinterpret_cast<__half*>(
        (reinterpret_cast<std::uintptr_t>(shift + ((tokens + 63) / 64) * 64 + 64) + 255) & ~std::uintptr_t(255));
    if (shi) *shi = s0;
    if (slo) *slo = s0 + std::size_t(tokens) * (cols / 32);
}

void launch_gemm_tc(const GemmArgs& g, void* workspace, std::size_t workspace_bytes, cudaStream_t s) {
    const int T = g.tokens, K = g.w.cols;
    if (!workspace || workspace_bytes < gemm_tc_workspace(T, K))
        throw std::invalid_argument("tensor-core projection workspace too small");
    __half *hi = nullptr, *lo = nullptr, *shi = nullptr, *slo = nullptr;
    int* shift = nullptr;
    gemm_tc_split_buffers(workspace, workspace_bytes, T, K, hi, lo, shift, &shi, &slo);
    // callers without an error flag get one in the workspace (never null)
    int* err = g.err ? g.err : shift + ((T + 63) / 64) * 64;
    // small batches of packed Q4_K rows (gemm_small_q4k_kernel): the stages
    // take 16- and 8-byte copies of the side arrays and activations
    const auto a16 = [](const void* p) { return reinterpret_cast<std::uintptr_t>(p) % 16 == 0; };
    const bool small_q4k = g.w.qsc && T <= 64 && g_small_batches && a16(g.w.qs) && g.w.qs_row % 16 == 0 &&
                           a16(g.w.qsc) && a16(g.w.qmin_hi) && a16(g.w.qmin_lo) && a16(g.w.qscale) &&
                           a16(g.w.qmin_shift) && a16(hi) && a16(lo) && a16(shi) && a16(slo);
    SmallWork wk{};
    if (small_q4k) {
        const int nt = T <= 8 ? 1 : T <= 16 ? 2 : T <= 32 ? 4 : 8;
        const int cb = nt <= 2 ? 2 : 1;  // blocks per chunk (small_ck)
        const int blocks = K / 256, chunks = (blocks + cb - 1) / cb;
        const bool split = g.epilogue != kSwiGLU;  // SwiGLU needs whole sums
        wk.row_tiles = (g.w.rows + kSmallRows - 1) / kSmallRows;
        wk.pairs = wk.row_tiles * (split ? chunks : 1);
        wk.slice_units = split ? cb * 8 : K / 32;
        wk.chunks = split ? 1 : chunks;
        // split partial sums are added into y: zero it before the split kernel,
        // so that the projection's predecessor on the stream is a kernel (its
        // programmatic launch then overlaps the weight copies with the split)
        if (split && chunks > 1 && g.epilogue == kStore)
            TVARA_CUDA(cudaMemset2DAsync(g.y, std::size_t(g.ldy) * 4, 0, std::size_t(g.w.rows) * 4, T, s));
    }
    if (!g.presplit) {
        if (reinterpret_cast<std::uintptr_t>(g.x) % 16 || g.ldx % 4 || K % 4)
            throw std::invalid_argument("tensor-core projection input must be 16-byte aligned rows");
        split_kernel<<<T, 256, 0, s>>>(g.x, g.ldx, K, hi, lo, shift, shi, slo);
        TVARA_LAUNCHED();
    }

    if (small_q4k) {
        // small batches: packed Q4_K rows on mma.sync, weights read once for all tokens
        const int nt = T <= 8 ? 1 : T <= 16 ? 2 : T <= 32 ? 4 : 8;
        const int atomic = wk.pairs > wk.row_tiles;
        switch (nt) {
#define TVARA_SMALL(N)                                                                                             \
    case N: {                                                                                                      \
        auto kernel = gemm_small_q4k_kernel<N>;                                                                    \
        constexpr int smem = int(small_smem_bytes<N>());                                                           \
        TVARA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));               \
        static const int per_sm = [&] {                                                                            \
            int n = 0;                                                                                             \
            TVARA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kSmallThreads * small_groups<N>(), smem)); \
            return n > 0 ? n : 1;                                                                                  \
        }();                                                                                                       \
        cudaLaunchConfig_t cfg = {};                                                                               \
        cfg.gridDim = dim3(std::min(wk.pairs, sm_count() * per_sm));                                               \
        cfg.blockDim = dim3(kSmallThreads * small_groups<N>());                                                    \
        cfg.dynamicSmemBytes = smem;                                                                               \
        cfg.stream = s;                                                                                            \
        cudaLaunchAttribute attr[1];                                                                               \
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                                           \
        attr[0].val.programmaticStreamSerializationAllowed = 1;                                                    \
        cfg.attrs = attr;                                                                                          \
        cfg.numAttrs = 1;                                                                                          \
        TVARA_CUDA(cudaLaunchKernelEx(&cfg, kernel, g.w, (const __half*)hi, (const __half*)lo, (const int*)shift,  \
                                      (const __half*)shi, (const __half*)slo, T, wk, g.y, g.ldy, g.epilogue,       \
                                      atomic));                                                                    \
        break;                                                                                                     \
    }
            TVARA_SMALL(1)
            TVARA_SMALL(2)
            TVARA_SMALL(4)
            TVARA_SMALL(8)
#undef TVARA_SMALL
        }
        TVARA_LAUNCHED();
        return;
    }
    if ((g.w.type == kQ8_0 || g.w.type == kQ4_0) && T <= kSmallQMaxTokens && g_small_batches && g.w.qs_row % 8 == 0) {
        // small batches: packed Q8_0 / Q4_0 rows on mma.sync, weights read once per 64 tokens
        const int nt = T <= 8 ? 1 : T <= 16 ? 2 : 4;
        const int groups = (T + 8 * nt - 1) / (8 * nt);
        const int row_tiles = (g.w.rows + kSmallRows - 1) / kSmallRows;
        int splits = 1;  // K slices of whole 256-element chunks
        if (g.epilogue != kSwiGLU)
            while (K % (splits * 2 * kSmallQChunk) == 0 && row_tiles * splits * groups < 3 * sm_count()) splits *= 2;
        if (splits > 1 && g.epilogue == kStore)
            TVARA_CUDA(cudaMemset2DAsync(g.y, std::size_t(g.ldy) * 4, 0, std::size_t(g.w.rows) * 4, T, s));
        const dim3 grid(row_tiles, splits, groups);
        const int kslice = K / splits;
        const int code = (g.w.type == kQ8_0 ? 0 : 16) + nt;
        switch (code) {
#define TVARA_SMALLQ(C, TY, N)                                                                                     \
    case C: {                                                                                                      \
        const int smem = int(smallq_smem_bytes<TY>(N));                                                            \
        TVARA_CUDA(cudaFuncSetAttribute(gemm_small_q8_kernel<TY, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)); \
        gemm_small_q8_kernel<TY, N><<<grid, kSmallThreads, smem, s>>>(g.w, hi, lo, shift, T, kslice, g.y, g.ldy,    \
                                                                      g.epilogue, splits > 1);                     \
        break;                                                                                                     \
    }
            TVARA_SMALLQ(1, kQ8_0, 1)
            TVARA_SMALLQ(2, kQ8_0, 2)
            TVARA_SMALLQ(4, kQ8_0, 4)
            TVARA_SMALLQ(17, kQ4_0, 1)
            TVARA_SMALLQ(18, kQ4_0, 2)
            TVARA_SMALLQ(20, kQ4_0, 4)
#undef TVARA_SMALLQ
        }
        TVARA_LAUNCHED();
        return;
    }
    const int row_tiles = (g.w.rows + kBM - 1) / kBM;
    const int steps = K / kBK;
    const bool q4k_form = g.w.qplane || g.w.qsc;
    // packed Q4_K rows: by default the one-CTA tensor-memory form or the
    // shared-memory form, whichever the tile plans make faster (below);
    // TVARA_Q4K_A=tmem / smem / pair forces one form (tests, comparisons)
    static const int q4k_a_form = [] {
        const char* v = std::getenv("TVARA_Q4K_A");
        if (v && std::strcmp(v, "smem") == 0) return 0;
        if (v && std::strcmp(v, "pair") == 0) return 2;
        if (v && std::strcmp(v, "tmem") == 0) return 3;
        return 1;
    }();
    const bool packed_q4k = !g.w.qplane && g.w.qsc;
    const bool pair = packed_q4k && q4k_a_form == 2 && sm_count() >= 2;
    bool tmem_a = packed_q4k && q4k_a_form >= 1;
    // the pair form's tiles are 256 rows, one per two SMs
    const int plan_rows = pair ? (g.w.rows + kPairRows - 1) / kPairRows : row_tiles;
    const bool can_split = g.epilogue != kSwiGLU;
    TilePlan plan = plan_tiles(plan_rows, T, steps, can_split, pair ? sm_count() / 2 : sm_count(),
                               pair ? kQ4kPairMaxN : tmem_a ? kQ4kpTmemMaxN : kMaxN,
                               tmem_a ? double(kQ4kpTmemMaxN + 48) : 0.0, q4k_form);
    if (tmem_a && !pair && q4k_a_form == 1) {
        // the tensor-memory form's K-step is ~1.35x faster than the shared-memory
        // form's at the same tile (measured on the 8B shapes), but its tiles stop
        // at 192 tokens; where 256-wide tiles with split K need far fewer K-steps
        // per SM (the 4096-row projections), the shared-memory form is faster
        const TilePlan ps = plan_tiles(row_tiles, T, steps, can_split, sm_count(), kMaxN, 0.0, true);
        auto per_sm = [&](const TilePlan& p) {
            const long long tiles = (long long)row_tiles * p.token_tiles * p.splits;
            return double((tiles + sm_count() - 1) / sm_count()) * double(steps / p.splits);
        };
        if (per_sm(plan) > 1.35 * per_sm(ps)) {
            tmem_a = false;
            plan = ps;
        }
    }
    if (q4k_form)  // whole 256-element blocks per split
        while (plan.splits > 1 && (steps / 8) % plan.splits) plan.splits /= 2;
    const int n_tile = plan.n_tile, token_tiles = plan.token_tiles, splits = plan.splits;
    TcArgs a;
    a.w = g.w;
    a.x_shift = shift;
    a.y = g.y;
    a.ldy = g.ldy;
    a.tokens = T;
    a.n_tile = n_tile;
    a.k_steps = steps / splits;
    a.epilogue = g.epilogue;
    a.atomic = splits > 1;
    a.idesc = (1u << 4) | (unsigned(n_tile >> 3) << 17) | (unsigned(kBM >> 4) << 24);
    a.err = err;
    if (!g.err) TVARA_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
    if (splits > 1 && g.epilogue == kStore)
        TVARA_CUDA(cudaMemset2DAsync(g.y, std::size_t(g.ldy) * 4, 0, std::size_t(g.w.rows) * 4, T, s));
    const CUtensorMap mh = make_map(hi, K, T, n_tile), ml = make_map(lo, K, T, n_tile);
    const dim3 grid(token_tiles, row_tiles, splits);
    if (q4k_form) {
        // Q4_K two-MMA kernel: splits whole 256-element blocks; y was zeroed above for split K
        if (steps % (8 * splits)) throw std::logic_error("Q4_K split does not divide the blocks");
        const int units = K / 32;  // sub-block sums written with the split
        const CUtensorMap mq = g.w.qplane ? make_map(reinterpret_cast<const __half*>(g.w.qplane), K, g.w.rows, kBM)
                                          : make_packed_map(g.w.qs, g.w.qs_row, g.w.rows,
                                                            tmem_a ? Q4kpForm<true>::kPkSteps : 1);
        const CUtensorMap mmh = make_map(reinterpret_cast<const __half*>(g.w.qmin_hi), units, g.w.rows, kBM);
        const CUtensorMap mml = make_map(reinterpret_cast<const __half*>(g.w.qmin_lo), units, g.w.rows, kBM);
        const CUtensorMap msh = make_map(shi, units, T, n_tile), msl = make_map(slo, units, T, n_tile);
        Q4kArgs qa;
        qa.t = a;
        qa.blocks = a.k_steps / 8;
        qa.min_steps = (units + kBK - 1) / kBK;
        TileSpace ts{token_tiles, row_tiles, splits, token_tiles * row_tiles * splits};
        const int smem = kStages * (2 * kATile + 2 * kBTileMax) + 1024 + 256;
        const int grid_n = std::min(ts.n_tiles, sm_count());
        if (g.w.qplane) {
            TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            tc_gemm_q4k_kernel<<<grid_n, kPersistThreads, smem, s>>>(mh, ml, mq, mmh, mml, msh, msl, qa, ts);
        } else {
            if (g.w.qs_row % 16 || reinterpret_cast<std::uintptr_t>(g.w.qs) % 16)
                throw std::invalid_argument("packed Q4_K rows must be 16-byte aligned");
            if (pair) {
                if (n_tile > kQ4kPairMaxN) throw std::logic_error("token tile too wide for the CTA-pair form");
                constexpr int smem_p = Q4kPairForm::smem_bytes();
                static_assert(smem_p <= 227 * 1024, "CTA-pair form exceeds shared memory");
                // each CTA of a pair loads half of the tile's tokens
                const CUtensorMap ph = make_map(hi, K, T, n_tile / 2), pl = make_map(lo, K, T, n_tile / 2);
                const CUtensorMap psh = make_map(shi, units, T, n_tile / 2), psl = make_map(slo, units, T, n_tile / 2);
                TileSpace pts{token_tiles, plan_rows, splits, token_tiles * plan_rows * splits};
                const int pairs = std::min(pts.n_tiles, sm_count() / 2);
                TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_q4k2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_p));
                tc_gemm_q4k2_kernel<<<2 * pairs, kQ4kpThreads, smem_p, s>>>(ph, pl, mq, psh, psl, qa, pts);
            } else if (tmem_a) {
                if (n_tile > kQ4kpTmemMaxN) throw std::logic_error("token tile too wide for the tensor-memory A form");
                constexpr int smem_p = Q4kpForm<true>::smem_bytes();
                static_assert(smem_p <= 227 * 1024, "tensor-memory A form exceeds shared memory");
                TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_q4kp_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                smem_p));
                tc_gemm_q4kp_kernel<true><<<grid_n, kQ4kpThreads, smem_p, s>>>(mh, ml, mq, mmh, mml, msh, msl, qa, ts);
            } else {
                constexpr int smem_p = Q4kpForm<false>::smem_bytes();
                static_assert(smem_p <= 227 * 1024, "shared-memory A form exceeds shared memory");
                TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_q4kp_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                smem_p));
                tc_gemm_q4kp_kernel<false><<<grid_n, kQ4kpThreads, smem_p, s>>>(mh, ml, mq, mmh, mml, msh, msl, qa, ts);
            }
        }
        TVARA_LAUNCHED();
        return;
    }
    if (g.w.plane_hi && g.w.plane_lo) {
        const CUtensorMap pa = make_map(reinterpret_cast<const __half*>(g.w.plane_hi), K, g.w.rows, kBM);
        const CUtensorMap pb = make_map(reinterpret_cast<const __half*>(g.w.plane_lo), K, g.w.rows, kBM);
        if (g_tc_persistent) {
            TileSpace ts{token_tiles, row_tiles, splits, token_tiles * row_tiles * splits};
            const int smem = kStages * (2 * kATile + 2 * kBTileMax) + 1024 + 256;
            TVARA_CUDA(cudaFuncSetAttribute(tc_gemm_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            tc_gemm_persist_kernel<<<std::min(ts.n_tiles, sm_count()), kPersistThreads, smem, s>>>(mh, ml, pa, pb, a, ts);
            TVARA_LAUNCHED();
        } else {
            run_tc<kPlanes>(mh, ml, pa, pb, a, grid, s);
        }
        return;
    }
    switch (g.w.type) {
        case kQ4_K: run_tc<kQ4_K>(mh, ml, mh, ml, a, grid, s); break;
        case kQ4_0: run_tc<kQ4_0>(mh, ml, mh, ml, a, grid, s); break;
        case kQ8_0: run_tc<kQ8_0>(mh, ml, mh, ml, a, grid, s); break;
        case kF16: run_tc<kF16>(mh, ml, mh, ml, a, grid, s); break;
        case kF32: run_tc<kF32>(mh, ml, mh, ml, a, grid, s); break;
        default: throw std::invalid_argument("unsupported projection type");
    }
}

void set_tc_min_tokens(int n) { g_tc_min_tokens = n; }

void launch_projection(const GemmArgs& a, void* workspace, std::size_t workspace_bytes, cudaStream_t s) {
    if (workspace && gemm_tc_supported(a.w, a.tokens)) launch_gemm_tc(a, workspace, workspace_bytes, s);
    else launch_gemv(a, s);
}

}  // namespace tvara
