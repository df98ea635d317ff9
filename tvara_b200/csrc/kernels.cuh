// Kernel launchers of the B200 decode/prefill engine (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.hpp"

namespace tvara {

// ---- epilogues of the projection kernels --------------------------------
enum Epilogue : int {
    kStore = 0,   // y[t][c] = acc
    kAdd = 1,     // y[t][c] += acc            (residual add, o_proj / down_proj)
    kSwiGLU = 2,  // rows (2i, 2i+1) = (gate_i, up_i): y[t][i] = silu(gate)*up
};

struct GemmArgs {
    DeviceMatrix w;
    const float* x = nullptr;   // [tokens][ldx] F32 activations
    int ldx = 0;
    bool presplit = false;      // tensor-core path: x already split into the workspace (launch_rmsnorm_split)
    int tokens = 0;
    float* y = nullptr;         // [tokens][ldy]
    int ldy = 0;
    int epilogue = kStore;
    int* err = nullptr;         // device error flag (tensor-core path)
};

// y = epilogue(x . W^T): CUDA-core GEMV for small token counts.
void launch_gemv(const GemmArgs& a, cudaStream_t s);
// Tensor-core (tcgen05/TMEM) projection for larger token counts; falls
// back to nothing -- callers pick it only where gemm_tc_supported() holds.
bool gemm_tc_supported(const DeviceMatrix& w, int tokens);
void launch_gemm_tc(const GemmArgs& a, void* workspace, std::size_t workspace_bytes, cudaStream_t s);
std::size_t gemm_tc_workspace(int max_tokens, int max_cols);
// Where the tensor-core path keeps the split activations of `tokens` rows of
// width `cols` in its workspace (hi, lo FP16 [tokens][cols], per-row shift).
// (hi, lo [tokens][cols], shift [tokens], and the sub-block sums shi, slo
// [tokens][cols / 32] of the Q4_K min term, written when cols % 32 == 0)
void gemm_tc_split_buffers(void* workspace, std::size_t workspace_bytes, int tokens, int cols, __half*& hi,
                           __half*& lo, int*& shift, __half** shi = nullptr, __half** slo = nullptr);
// Choose and run the projection (GEMV below the crossover, tensor cores above).
void launch_projection(const GemmArgs& a, void* workspace, std::size_t workspace_bytes, cudaStream_t s);

// ---- block unpack / repack ----------------------------------------------
// GGUF blocks of `type` -> F32, bit-exact with the reference's dequantisers.
void launch_dequantize(int type, const void* blocks, std::size_t nblocks, float* out, cudaStream_t s);
// GGUF rows [rows][row bytes] -> engine split layout (qs, meta).
void launch_repack(int type, const void* gguf, int rows, int cols, std::uint8_t* qs, std::uint8_t* meta,
                   cudaStream_t s);
// Sets *flag when any dequantised value of the matrix is not finite.
void launch_finite_check(const DeviceMatrix& w, int* flag, cudaStream_t s);
// Per-row power-of-two scale of the tensor-core split (DeviceMatrix::row_shift).
void launch_row_shift(const DeviceMatrix& w, signed char* out, cudaStream_t s);
// Fills hi / lo ([rows][cols] FP16 each) with the exact split of every
// value times 2^row_shift (the tensor-core planes of DeviceMatrix).
void launch_planes(const DeviceMatrix& w, std::uint16_t* hi, std::uint16_t* lo, cudaStream_t s);
// Q4_K tensor-core form (DeviceMatrix::qplane ...) in `storage` of
// q4k_planes_bytes; sets the matrix's pointers.
std::size_t q4k_planes_bytes(int rows, int cols);
void launch_q4k_planes(DeviceMatrix& w, void* storage, cudaStream_t s);
// The packed Q4_K form (DeviceMatrix::qsc ...): side arrays only, about 0.16
// bytes per weight, the codes staying in the packed rows.
std::size_t q4k_packed_form_bytes(int rows, int cols);
void launch_q4k_packed_form(DeviceMatrix& w, void* storage, cudaStream_t s);
// Minimum token count routed to the tensor-core projection.
void set_tc_min_tokens(int n);

// ---- elementwise ----------------------------------------------------------
// x[t] = row tokens[t] of the embedding, dequantised.
// ids (optional): token id plane of the KV pool, ids[blk[t] * tpb + slot[t]] = tokens[t]
void launch_embed(const DeviceMatrix& emb, const int* tokens, int n, float* x, int ldx, cudaStream_t s,
                  int* ids = nullptr, const int* blk = nullptr, const int* slot = nullptr, int tpb = 0);
// out[i] = (x[rows[i]] * inv_rms) * w ; rows == nullptr means i.
void launch_rmsnorm(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps,
                    float* out, int ldo, cudaStream_t s);
// launch_rmsnorm that also writes the output's exact hi/lo split into the
// tensor-core workspace (then a projection with presplit skips its split);
// out may be null.
void launch_rmsnorm_split(const float* x, int ldx, const int* rows, int n, int dim, const float* w, float eps,
                          float* out, int ldo, void* tc_workspace, std::size_t tc_workspace_bytes, cudaStream_t s);

struct RopeArgs {
    const float* qkv = nullptr;  // [T][ldqkv]: q (hq*d) | k (hkv*d) | v (hkv*d)
    int ldqkv = 0;
    float* q = nullptr;          // [T][hq*d] rotated queries
    int tokens = 0, hq = 0, hkv = 0, dim = 0;
    bool interleaved = false;
    const float* cosines = nullptr;  // [context][dim/2]
    const float* sines = nullptr;
    const int* positions = nullptr;  // [T]
    const int* slot_block = nullptr; // [T] physical block of the token's position
    const int* slot_index = nullptr; // [T] slot within the block
    void* kv = nullptr;              // pool base
    int kv_f16 = 0;
    int kv_i8 = 0;                   // int8 per token-head with F32 scales (kv_scales)
    float* kv_scales = nullptr;      // [element offset of a row / dim] for kv_i8
    long long block_stride = 0, layer_offset = 0, kind_stride = 0;  // elements
    int tpb = 0;
    int max_blocks = 0;
    int* err = nullptr;
};
// Rotates q and k at each token's position and writes k, v into the pool.
// int8 pools: each (token, KV head) row is stored as the reference's
// quantized_kv encode (python/tvara/quantized_kv.py:21-30): scale = max|x| /
// 127 (1 for a zero row, the smallest subnormal if that underflows),
// values rint(x / scale) clipped to [-127, 127]; a non-finite row sets the
// error flag (3).  Dynamic shared memory: rope_kv_smem bytes.
std::size_t rope_kv_smem(const RopeArgs& a);
// The same encode on n rows of d floats (codes [n][d], scales [n]).
void launch_kv_quantize(const float* rows, int n, int d, signed char* codes, float* scales, int* err, cudaStream_t s);
void launch_rope_kv(const RopeArgs& a, cudaStream_t s);

// g[i] = g[i] * (sigmoid(g[i]) * u[i]) for separate gate/up projections.
void launch_swiglu(float* g, const float* u, long long n, cudaStream_t s);

// ---- paged attention -------------------------------------------------------
struct AttnArgs {
    const float* q = nullptr;  // [T][hq*d]
    float* out = nullptr;      // [T][hq*d]
    const void* kv = nullptr;
    int kv_f16 = 0;
    int kv_i8 = 0;                    // int8 rows with F32 scales
    const float* kv_scales = nullptr; // row r (element offset / dim) scale
    int hq = 0, hkv = 0, dim = 0, tpb = 0;
    long long block_stride = 0, layer_offset = 0, kind_stride = 0;  // elements
    const int* tables = nullptr;  // concatenated physical block ids
    const int4* work = nullptr;   // {token, table offset, pos begin, pos end}
    const int* work_part = nullptr;  // partial slot per work item, -1 = whole range
    int n_work = 0;
    float* partial = nullptr;     // [n_parts][hq][dim+2]
    const int4* combine = nullptr; // {token, first part, part count, 0}
    int n_combine = 0;
    int max_blocks = 0;
    int* err = nullptr;
    // chunks of consecutive query rows of one sequence, run by the chunk
    // kernel: {first row, table offset, visible positions of the first row
    // (row r sees one more per r), rows}
    const int4* chunk_work = nullptr;
    int n_chunk = 0;
};
void launch_attention(const AttnArgs& a, cudaStream_t s);
// Rows per chunk the chunk kernels take for this shape (kv_kind 0 = F32 or
// 1 = F16 pool, head_dim 64 or 128, 1..8 query heads per KV head, blocks of a
// multiple of 16 slots), 0 when they do not apply (int8 pools: kv_kind 2).
int attention_chunk_rows(int kv_kind, int dim, int group, int tpb);

// ---- output ---------------------------------------------------------------
// argmax of each row (first index of the maximum; NaN counts as maximal);
// with finite_check, rows holding a NaN or infinity report 0xFFFFFFFF.
void launch_argmax(const float* logits, int rows, int vocab, unsigned* out, bool finite_check, cudaStream_t s);
// The same over a vocabulary split across ranks: each rank reduces columns
// [col0, col0 + cols) of its rows (row stride ld) to argmax_part_bytes()
// per row; the gathered parts [rank][row] merge into out.
std::size_t argmax_part_bytes();
void launch_argmax_part(const float* logits, int rows, int ld, int cols, int col0, void* parts, cudaStream_t s);
void launch_argmax_merge(const void* parts, int rows, int ranks, unsigned* out, bool finite_check, cudaStream_t s);
// Copies whole KV blocks (copy-on-write): pairs of (from, to) block ids.
void launch_block_copy(void* kv, long long block_bytes, const int2* pairs, int n, cudaStream_t s);
// The same pairs over the token id plane ([block][per_block] ints).
void launch_id_copy(int* ids, int per_block, const int2* pairs, int n, cudaStream_t s);

// Device-side logit post-processing (k_sample.cu): penalties from each row's
// token history, the token mask, finiteness checks, argmax and top-k.
constexpr int kSampleMaxK = 64;
enum { kSampleNonfiniteLogits = 1, kSampleNonfiniteAdjusted = 2, kSampleNoneAllowed = 4 };
struct SampleJob {
    const float* logits = nullptr;  // row r at logits + r * ld
    long long ld = 0;
    int rows = 0, vocab = 0;
    // history of row r: flat hist[hoff[r] ..), or through the KV pool's token
    // ids: ids[tables[toff[r] + i / tpb] * tpb + i % tpb]; hlen[r] tokens
    const int* hist = nullptr;
    const long long* hoff = nullptr;
    const int* ids = nullptr;
    const int* tables = nullptr;
    const int* toff = nullptr;
    int tpb = 1;
    const int* hlen = nullptr;
    int hist_cap = 1;                  // power of two >= every hlen
    const double* params = nullptr;    // [rows][3]: repetition, frequency, presence
    const unsigned* allowed = nullptr; // [rows][words] bitmask or null
    int words = 0;
    int top_k = 0;
    double* pen = nullptr;             // scratch [rows][pen_stride >= hist_cap]
    long long pen_stride = 0;
    unsigned* argmax = nullptr;        // [rows]
    int* status = nullptr;             // [rows] kSample* bits
    double* top_val = nullptr;         // [rows][top_k]
    unsigned* top_id = nullptr;        // [rows][top_k]
};
std::size_t sample_smem_bytes(int vocab, int hist_cap);
void launch_sample(const SampleJob& j, cudaStream_t s);

}  // namespace tvara
