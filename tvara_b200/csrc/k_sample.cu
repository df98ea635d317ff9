// Device-side logit post-processing: the sampler of the reference's
// NativeModel.iter_tokens (python/tvara/native.py:301-336) up to its random
// draw, for many rows at once.  Per row, in float64 with the same IEEE
// operations as the numpy code:
//   adjusted = logits (as float64)
//   seen tokens:  adjusted = adjusted >= 0 ? adjusted / repetition : adjusted * repetition
//   every token:  adjusted -= count * frequency + seen * presence
//   masked      = allowed ? adjusted : -inf          (token_masks.py:228-241)
// and then the first index of the maximum of `masked` (np.argmax) and the
// top-k candidates of `masked` by value, ties by index.  Status bits record
// the reference's checks: non-finite model logits (native.py:304-305),
// non-finite adjusted logits (native.py:312-313), no allowed token
// (token_masks.py:237-238).
//
// The history of a row -- the tokens already in its sequence -- is read
// through its block table from the KV pool's token id plane (or from a flat
// array), sorted in shared memory, and each distinct token's penalised value
// is kept at its first position, so a full-vocabulary pass costs one float
// load, one bit test and, for seen tokens only, a binary search.
#include <math_constants.h>

#include <cstdint>
#include <stdexcept>

#include "kernels.cuh"

namespace tvara {
namespace {

constexpr int kSampleThreads = 512;
constexpr int kSampleWarps = kSampleThreads / 32;

__device__ __forceinline__ unsigned long long select_key(double v) {
    // smaller key = larger value (the selection keeps the smallest keys); -0 and +0 share one key
    unsigned long long u = static_cast<unsigned long long>(__double_as_longlong(v));
    if ((u << 1) == 0) u = 0;
    const unsigned long long asc = (u >> 63) ? ~u : (u | 0x8000000000000000ull);
    return ~asc;
}

struct RowView {
    const float* lg;
    const unsigned* hist;  // sorted history in shared memory
    const unsigned* seen;  // bitmap of seen tokens in shared memory
    const double* pen;     // penalised value at each distinct token's first history position
    const unsigned* allowed;
    int n;
    double fr, pr;
    // adjusted value (before the mask)
    __device__ __forceinline__ double adjusted(int t) const {
        if ((seen[t >> 5] >> (t & 31)) & 1u) {
            int lo = 0, hi = n;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (hist[mid] < unsigned(t)) lo = mid + 1;
                else hi = mid;
            }
            return pen[lo];
        }
        // count 0, not seen: adjusted - (0 * frequency + 0 * presence)
        return __dsub_rn(double(lg[t]), __dadd_rn(__dmul_rn(0.0, fr), __dmul_rn(0.0, pr)));
    }
    __device__ __forceinline__ bool is_allowed(int t) const {
        return !allowed || ((allowed[t >> 5] >> (t & 31)) & 1u);
    }
    __device__ __forceinline__ double masked(int t) const {
        return is_allowed(t) ? adjusted(t) : -CUDART_INF;
    }
};

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleJob j) {
    extern __shared__ __align__(16) unsigned char sample_smem[];
    unsigned* s_hist = reinterpret_cast<unsigned*>(sample_smem);  // [hist_cap]
    unsigned* s_seen = s_hist + j.hist_cap;                        // [ceil(vocab / 32)]
    unsigned* s_bins = s_seen + (j.vocab + 31) / 32;               // [4096]
    __shared__ unsigned long long s_key[64];
    __shared__ double s_val[64];
    __shared__ unsigned s_idx[64];
    __shared__ double s_best[kSampleWarps];
    __shared__ int s_besti[kSampleWarps];
    __shared__ unsigned s_wsum[kSampleWarps];
    __shared__ unsigned s_digit, s_before, s_count;
    __shared__ int s_taken, s_eq_taken;

    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = j.vocab;
    const float* lg = j.logits + (long long)r * j.ld;
    const int n = j.hlen[r];
    const double rep = j.params[3 * r], fr = j.params[3 * r + 1], pr = j.params[3 * r + 2];
    const unsigned* allowed = j.allowed ? j.allowed + (long long)r * j.words : nullptr;
    double* pen = j.pen + (long long)r * j.pen_stride;

    // ---- model logits finite (checked before any adjustment)
    int bad = 0;
    for (int t = tid; t < V; t += kSampleThreads) bad |= !isfinite(lg[t]);
    bad = __syncthreads_or(bad);

    // ---- history, sorted
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += kSampleThreads) {
        unsigned id = 0xFFFFFFFFu;
        if (i < n) {
            int v;
            if (j.hist) v = j.hist[j.hoff[r] + i];
            else v = j.ids[(long long)j.tables[j.toff[r] + i / j.tpb] * j.tpb + i % j.tpb];
            if (v >= 0 && v < V) id = unsigned(v);  // reserved positions (-1) hold no token
        }
        s_hist[i] = id;
    }
    for (int i = tid; i < (V + 31) / 32; i += kSampleThreads) s_seen[i] = 0;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1)
        for (int m = k >> 1; m > 0; m >>= 1) {
            for (int i = tid; i < P; i += kSampleThreads) {
                const int o = i ^ m;
                if (o > i) {
                    const unsigned a = s_hist[i], b = s_hist[o];
                    if (((i & k) == 0) == (a > b)) {
                        s_hist[i] = b;
                        s_hist[o] = a;
                    }
                }
            }
            __syncthreads();
        }
    // ---- penalised value of each distinct token, at its first position
    for (int i = tid; i < n; i += kSampleThreads) {
        const unsigned t = s_hist[i];
        if (t == 0xFFFFFFFFu || (i > 0 && s_hist[i - 1] == t)) continue;
        int c = 1;
        while (i + c < n && s_hist[i + c] == t) ++c;
        double v = double(lg[t]);
        v = v >= 0.0 ? __ddiv_rn(v, rep) : __dmul_rn(v, rep);
        v = __dsub_rn(v, __dadd_rn(__dmul_rn(double(c), fr), __dmul_rn(1.0, pr)));
        pen[i] = v;
        atomicOr(&s_seen[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
    RowView row{lg, s_hist, s_seen, pen, allowed, n, fr, pr};

    // ---- argmax of the masked values; adjusted values finite; any token allowed
    double best = -CUDART_INF;
    int besti = 0x7FFFFFFF, nonfinite = 0, any = 0;
    for (int t = tid; t < V; t += kSampleThreads) {
        const double a = row.adjusted(t);
        nonfinite |= !isfinite(a);
        const bool ok = row.is_allowed(t);
        any |= ok;
        const double v = ok ? a : -CUDART_INF;
        if (v > best || (v == best && t < besti)) {
            best = v;
            besti = t;
        }
    }
    for (int o = 16; o; o >>= 1) {
        const double ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ob > best || (ob == best && oi < besti)) {
            best = ob;
            besti = oi;
        }
    }
    if (lane == 0) {
        s_best[warp] = best;
        s_besti[warp] = besti;
    }
    nonfinite = __syncthreads_or(nonfinite);
    any = __syncthreads_or(any);
    if (tid == 0) {
        for (int w = 1; w < kSampleWarps; ++w)
            if (s_best[w] > best || (s_best[w] == best && s_besti[w] < besti)) {
                best = s_best[w];
                besti = s_besti[w];
            }
        j.argmax[r] = unsigned(besti);
        j.status[r] = (bad ? kSampleNonfiniteLogits : 0) | (!bad && nonfinite ? kSampleNonfiniteAdjusted : 0) |
                      (any ? 0 : kSampleNoneAllowed);
    }
    const int K = j.top_k;
    if (K <= 0) return;

    // ---- top-k: radix selection of the K smallest keys (12-bit digits from the top)
    unsigned long long prefix = 0, pmask = 0;
    int need = K;
    for (int pass = 0; pass < 6; ++pass) {
        const int shift = pass < 5 ? 52 - 12 * pass : 0;
        const unsigned nb = pass < 5 ? 4096u : 16u;
        for (unsigned i = tid; i < nb; i += kSampleThreads) s_bins[i] = 0;
        __syncthreads();
        for (int t = tid; t < V; t += kSampleThreads) {
            const unsigned long long key = select_key(row.masked(t));
            if ((key & pmask) == prefix) atomicAdd(&s_bins[(key >> shift) & (nb - 1)], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            const unsigned per = (nb + 31) / 32;
            const unsigned b0 = min(nb, lane * per), b1 = min(nb, (lane + 1) * per);
            unsigned local = 0;
            for (unsigned b = b0; b < b1; ++b) local += s_bins[b];
            unsigned incl = local;
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const unsigned excl = incl - local;
            const unsigned hit = __ballot_sync(0xffffffffu, incl >= unsigned(need) && excl < unsigned(need));
            if (hit && lane == __ffs(hit) - 1) {
                unsigned before = excl;
                for (unsigned b = b0; b < b1; ++b) {
                    if (before + s_bins[b] >= unsigned(need)) {
                        s_digit = b;
                        s_before = before;
                        s_count = s_bins[b];
                        break;
                    }
                    before += s_bins[b];
                }
            }
        }
        __syncthreads();
        need -= int(s_before);
        prefix |= (unsigned long long)s_digit << shift;
        pmask |= (unsigned long long)(nb - 1) << shift;
        const bool exact = int(s_count) == need;  // the whole bin is taken
        __syncthreads();
        if (exact) break;
    }
    // ---- collect: every key below the prefix, and the first `need` at it by index
    if (tid == 0) {
        s_taken = 0;
        s_eq_taken = 0;
    }
    __syncthreads();
    for (int base = 0; base < V; base += kSampleThreads) {
        const int t = base + tid;
        bool below = false, eq = false;
        unsigned long long key = 0;
        double v = 0.0;
        if (t < V) {
            v = row.masked(t);
            key = select_key(v);
            below = (key & pmask) < prefix;
            eq = (key & pmask) == prefix;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) s_wsum[warp] = __popc(bal);
        __syncthreads();
        int off = 0, tot = 0;
        for (int w = 0; w < kSampleWarps; ++w) {
            if (w < warp) off += int(s_wsum[w]);
            tot += int(s_wsum[w]);
        }
        const int rank = s_eq_taken + off + __popc(bal & ((1u << lane) - 1u));
        if (below || (eq && rank < need)) {
            const int slot = atomicAdd(&s_taken, 1);
            if (slot < 64) {
                s_key[slot] = key;
                s_val[slot] = v;
                s_idx[slot] = unsigned(t);
            }
        }
        __syncthreads();
        if (tid == 0) s_eq_taken += tot;
        __syncthreads();
    }
    // ---- order the K candidates: value descending, index ascending
    if (tid < 64 && tid >= K) {
        s_key[tid] = ~0ull;
        s_idx[tid] = 0xFFFFFFFFu;
    }
    __syncthreads();
    for (int k = 2; k <= 64; k <<= 1)
        for (int m = k >> 1; m > 0; m >>= 1) {
            if (tid < 64) {
                const int o = tid ^ m;
                if (o > tid) {
                    const bool gt = s_key[tid] > s_key[o] || (s_key[tid] == s_key[o] && s_idx[tid] > s_idx[o]);
                    if (((tid & k) == 0) == gt) {
                        const unsigned long long tk = s_key[tid];
                        s_key[tid] = s_key[o];
                        s_key[o] = tk;
                        const double tv = s_val[tid];
                        s_val[tid] = s_val[o];
                        s_val[o] = tv;
                        const unsigned ti = s_idx[tid];
                        s_idx[tid] = s_idx[o];
                        s_idx[o] = ti;
                    }
                }
            }
            __syncthreads();
        }
    if (tid < K) {
        j.top_val[(long long)r * K + tid] = s_val[tid];
        j.top_id[(long long)r * K + tid] = s_idx[tid];
    }
}

}  // namespace

std::size_t sample_smem_bytes(int vocab, int hist_cap) {
    return std::size_t(hist_cap) * 4 + std::size_t((vocab + 31) / 32) * 4 + 4096 * 4;
}

void launch_sample(const SampleJob& j, cudaStream_t s) {
    if (j.rows <= 0) return;
    if (j.top_k < 0 || j.top_k > kSampleMaxK || j.top_k > j.vocab)
        throw std::invalid_argument("top-k candidates must be between 0 and 64 and at most the vocabulary");
    const std::size_t smem = sample_smem_bytes(j.vocab, j.hist_cap);
    if (smem > 200 * 1024) throw std::invalid_argument("device sampling: history or vocabulary too large");
    TVARA_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    sample_kernel<<<j.rows, kSampleThreads, smem, s>>>(j);
    TVARA_LAUNCHED();
}

}  // namespace tvara
