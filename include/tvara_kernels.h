/*
 * tvara_kernels -- kernel-level C ABI of the B200 engine (device pointers).
 *
 * These expose single hot-path kernels without a model handle, for callers
 * that manage their own device memory (and for the standalone GEMV and
 * attention benchmarks).  Pointers marked "device" are CUDA device memory of
 * the current device; `stream` is a cudaStream_t (NULL = legacy default).
 * Every function returns 0 on success and -1 on failure, with the message in
 * tvara_last_error() (include/tvara_capi.h).  Launches are asynchronous.
 */
#ifndef TVARA_KERNELS_H
#define TVARA_KERNELS_H
#include <stddef.h>
#include <stdint.h>

#include "tvara_capi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF storage types (reference core/include/tvara/gguf.hpp:152-170). */
enum { TVARA_F32 = 0, TVARA_F16 = 1, TVARA_Q4_0 = 2, TVARA_Q8_0 = 8, TVARA_Q4_K = 12 };

/* Replaces quant::dequantize_q8_0 / q4_0 / q4_k and half_to_float
 * (core/include/tvara/quant.hpp:14-84): `blocks` GGUF blocks (device) ->
 * F32 (device), bit-identical to the reference. */
TVARA_API int tvara_dequantize(int type, const void* blocks, size_t nblocks, float* out, void* stream);

/* Bytes of the engine's packed layout for a [rows][cols] matrix: the codes of
 * every row (16-byte aligned rows), then the block headers, then one signed
 * byte per row (the power-of-two scale of the tensor-core path), each part at
 * a 256-byte aligned offset.  Q4_K rows (width a multiple of 256) are
 * followed by the side arrays the tensor-core path reads
 * beside the packed codes (sub-block scales, block scales, the split minima:
 * about 0.16 bytes per weight). */
TVARA_API size_t tvara_packed_bytes(int type, size_t rows, size_t cols);
/* GGUF rows (device) -> engine layout (device, tvara_packed_bytes long). */
TVARA_API int tvara_pack(int type, const void* gguf_rows, size_t rows, size_t cols, void* packed, void* stream);

/* Logit post-processing on the device (the sampler of
 * python/tvara/native.py:301-336 up to its random draw, for many rows):
 * logits F32 [rows][vocab] (device); the token history of row r is
 * history[history_offsets[r] .. history_offsets[r+1]) (history device,
 * offsets host, at most 16384 tokens a row); per-row repetition / frequency /
 * presence (host, NULL = 1, 0, 0); allowed (device [rows][ceil(vocab/32)]
 * bitmask, NULL = all).  Outputs on the device: argmax [rows] of the
 * adjusted, masked float64 logits, status [rows] (bit 1: non-finite model
 * logits, 2: non-finite adjusted logits, 4: no allowed token), and the
 * top_k (<= 64) largest values with their ids [rows][top_k] (value
 * descending, ties by index).  `workspace` of tvara_sample_workspace bytes. */
TVARA_API size_t tvara_sample_workspace(size_t rows, size_t max_history);
TVARA_API int tvara_sample_logits(const float* logits, size_t rows, size_t vocab, const int32_t* history,
                                  const uint64_t* history_offsets, const double* repetition, const double* frequency,
                                  const double* presence, const uint32_t* allowed, uint32_t top_k, uint32_t* argmax,
                                  int32_t* status, double* top_values, uint32_t* top_ids, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* The int8 KV encode of TVARA_KV_I8 pools (python/tvara/quantized_kv.py:
 * 21-30, QuantizedKV.encode): rows F32 [n][dim] (device) -> codes int8
 * [n][dim] and scales F32 [n] (device).  A non-finite row fails with
 * "Nonfinite KV input" (the call synchronises the stream to report it). */
TVARA_API int tvara_kv_quantize(const float* rows, size_t n, size_t dim, int8_t* codes, float* scales, void* stream);

/* Device scratch tvara_quant_matmul needs for `tokens` rows of width `cols`
 * (0 when the call runs on the CUDA-core path, at most 4 tokens). */
TVARA_API size_t tvara_quant_matmul_workspace(size_t cols, size_t tokens);
/* Replaces quant::matvec_f32 over dequantised weights / Matrix::multiply and
 * prefill_reference (quant.hpp:163-196, prefill.hpp:12-18):
 * y[t][r] = sum_k W[r][k] * x[t][k] for t < tokens, W packed (device), x and y
 * F32 row-major (device).  Up to 4 tokens: CUDA-core GEMV with the weights
 * dequantised in registers.  More: tcgen05 tensor cores on an exact hi+lo
 * FP16 split of both operands (F32 accumulation); needs `workspace`, and x
 * 16-byte aligned (cols is a multiple of 32 there). */
TVARA_API int tvara_quant_matmul(int type, const void* packed, size_t rows, size_t cols, const float* x,
                                 size_t tokens, float* y, void* workspace, size_t workspace_bytes, void* stream);

/* Paged GQA attention, replacing fused_paged_attention /
 * fused_prompt_attention (core/include/tvara/attention.hpp:57-89) for many
 * query rows at once.  Query row i attends to positions [0, visible[i]) of its
 * block list tables[table_offset[i] ..]; query head h reads KV head
 * h / (heads / kv_heads).  Pool layout (elements of kv_dtype): block b, layer
 * l, kind (0 K, 1 V), KV head g, slot s, element e at
 *   ((((b*layers + l)*2 + kind)*kv_heads + g)*block_tokens + s)*head_dim + e. */
typedef struct tvara_attention_args {
    uint32_t struct_size;       /* sizeof(tvara_attention_args) */
    uint32_t kv_dtype;          /* TVARA_KV_F32, TVARA_KV_F16 or TVARA_KV_I8 (needs kv_scales) */
    uint32_t heads, kv_heads, head_dim, block_tokens;
    uint32_t layers, layer;
    size_t max_blocks;
    size_t n_queries;
    const float* q;             /* device [n_queries][heads*head_dim] */
    float* out;                 /* device [n_queries][heads*head_dim] */
    const void* pool;           /* device KV pool */
    const int32_t* tables;      /* host: concatenated block ids */
    size_t tables_len;
    const uint32_t* table_offset; /* host [n_queries] */
    const uint32_t* visible;      /* host [n_queries], each >= 1 */
    /* TVARA_KV_I8: device F32 scale of each pool row (element offset / head_dim);
     * callers of the shorter struct (struct_size up to `visible`) get F32/F16 only */
    const float* kv_scales;
} tvara_attention_args;

/* Device scratch (bytes) tvara_paged_attention needs for these arguments;
 * 0 with an error for invalid arguments, including a block id outside
 * [0, max_blocks) in any block a query reads. */
TVARA_API size_t tvara_paged_attention_workspace(const tvara_attention_args* args);
/* Runs the attention; workspace is device memory of at least the size above.
 * The call uploads the block tables and work list from host memory and, after
 * the kernels, reads their error word back, so it returns only when the
 * attention has finished on `stream`; a device-side error (a copy wait that
 * timed out) returns -1 with its text.  Not capturable into a CUDA graph: a
 * capturing stream is refused with an error before anything is enqueued. */
TVARA_API int tvara_paged_attention(const tvara_attention_args* args, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* No counterpart in the reference (its attention runs on the CPU).  The same
 * attention as tvara_paged_attention, with its scratch in a fixed area inside
 * this library (tvara_paged_attention_noalloc_max() bytes per device, 16 MiB)
 * instead of caller memory, for callers that cannot allocate device memory at
 * the call: FFI hosts with no device allocator, code whose device memory
 * belongs to another framework's allocator, code that must not pay
 * cudaMalloc's device-wide synchronisation.  It allocates nothing.  Arguments
 * needing more scratch than the maximum (tvara_paged_attention_workspace) are
 * rejected with an error and nothing is launched.  The first call on a device,
 * with that device current, resolves the scratch address.  Synchronous on
 * `stream` and not capturable, as tvara_paged_attention; device-side errors
 * are returned the same way.  One scratch per device: calls overlapping on one
 * device (other streams or threads) race and must be serialised by the
 * caller. */
TVARA_API size_t tvara_paged_attention_noalloc_max(void);
TVARA_API int tvara_paged_attention_noalloc(const tvara_attention_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TVARA_KERNELS_H */
