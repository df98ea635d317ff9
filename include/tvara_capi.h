/*
 * tvara_capi -- C ABI of the B200 decode/prefill engine.
 *
 * The first eleven functions replace, with identical signatures and
 * semantics, the reference engine's ABI in core/include/tvara/c_api.h:13-24
 * (implemented in core/src/c_api.cpp:38-78), so the reference's
 * python/tvara/native.py (NativeModel) and speculative.py bind this library
 * unchanged through TVARA_LIBRARY.  Everything after them is additive.
 *
 * Conventions (as in the reference): every call clears the calling thread's
 * error string first; failures return NULL / 0 / -1 and leave a message
 * readable with tvara_last_error() until the next call on that thread.  One
 * mutex per handle serialises the sequence and step calls.  Output buffers
 * are caller-owned host memory; logits are F32 row-major [rows, vocab].
 */
#ifndef TVARA_CAPI_H
#define TVARA_CAPI_H
#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define TVARA_API __declspec(dllexport)
#else
#define TVARA_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tvara_model tvara_model;

/* ---- reference ABI (core/include/tvara/c_api.h:13-24) ------------------ */

/* c_api.h:13 / c_api.cpp:38-43.  Loads a Llama GGUF (F32, F16, Q4_0, Q8_0,
 * Q4_K tensors) onto the current CUDA device, keeping quantised blocks packed
 * in HBM, with a paged KV pool of max_blocks blocks of block_tokens positions
 * (F32 KV, one GPU).  NULL on error. */
TVARA_API tvara_model* tvara_model_open(const char* utf8_path, size_t max_blocks, size_t block_tokens);
/* c_api.h:14.  Releases the handle and its device memory; NULL-safe. */
TVARA_API void tvara_model_close(tvara_model* model);
/* c_api.h:15-16.  0 with "closed model" for a NULL handle. */
TVARA_API size_t tvara_model_vocab_size(tvara_model* model);
TVARA_API size_t tvara_model_context_size(tvara_model* model);
/* c_api.h:17.  Thread-local message of the last failed call. */
TVARA_API const char* tvara_last_error(void);
/* c_api.h:18.  JSON object of every GGUF metadata key, serialised as the
 * reference does (c_api.cpp:19-41); owned by the handle. */
TVARA_API const char* tvara_model_metadata(tvara_model* model);
/* c_api.h:19.  New empty sequence; ids start at 1; 0 on error. */
TVARA_API uint64_t tvara_sequence_create(tvara_model* model);
/* c_api.h:20.  Appends one token and writes its vocab logits; count must
 * equal the vocabulary.  All-or-nothing: on failure the sequence is
 * unchanged.  0 / -1. */
TVARA_API int tvara_sequence_decode(tvara_model* model, uint64_t sequence, uint32_t token, float* logits,
                                    size_t count);
/* c_api.h:21.  Releases the sequence's KV blocks.  0 / -1. */
TVARA_API int tvara_sequence_drop(tvara_model* model, uint64_t sequence);
/* c_api.h:22 / c_api.cpp:63-72.  Appends token_count tokens of one sequence
 * (a prefill chunk or a speculative verify) and writes every row's logits;
 * count must equal token_count*vocab.  On failure the sequence is truncated
 * back to its entry length.  0 / -1. */
TVARA_API int tvara_sequence_decode_batch(tvara_model* model, uint64_t sequence, const uint32_t* tokens,
                                          size_t token_count, float* logits, size_t count);
/* c_api.h:24.  Shortens a sequence (never extends it).  0 / -1. */
TVARA_API int tvara_sequence_truncate(tvara_model* model, uint64_t sequence, size_t length);

/* ---- additive: open options ------------------------------------------- */

/* TVARA_KV_I8: the reference's experimental per token-head int8 KV
 * (python/tvara/quantized_kv.py): int8 codes plus one F32 scale per
 * (token, KV head) row; lossy against the F32 KV of the served path. */
enum { TVARA_KV_F32 = 0, TVARA_KV_F16 = 1, TVARA_KV_I8 = 2 };

typedef struct tvara_open_options {
    uint32_t struct_size;      /* sizeof(tvara_open_options) */
    int32_t device;            /* CUDA ordinal; -1 keeps the current device */
    uint32_t kv_dtype;         /* TVARA_KV_F32 (reference numerics), TVARA_KV_F16 or TVARA_KV_I8 */
    uint32_t max_step_tokens;  /* tokens per device step (scratch sizing); 0 = 2048 */
    uint32_t tp_rank;          /* tensor-parallel rank of this handle */
    uint32_t tp_size;          /* tensor-parallel group size; 0 or 1 = no TP */
    const void* nccl_id;       /* 128-byte ncclUniqueId shared by the group (tp_size > 1) */
    uint32_t weight_planes;    /* tensor-core forms of the projections for batches of >= 5 tokens:
                                  Q4_K rows (width a multiple of 256) read packed, with
                                  side arrays of sub-block scales, block scales and minima (about
                                  0.16 bytes per weight), other types as exact FP16 hi/lo planes of
                                  their values (4 bytes per weight, like the reference's F32
                                  expansion).  0 = when they fit beside the KV pool, 1 = always,
                                  2 = never, 3 = hi/lo planes for every type, when they fit, 4 = as
                                  0 with Q4_K rows as a prebuilt FP16 plane of sc*q (2 bytes per
                                  weight).  Callers built against the shorter struct get 0. */
} tvara_open_options;

/* tvara_model_open with options; NULL options equal tvara_model_open.
 * struct_size may be that of an earlier, shorter version of the struct. */
TVARA_API tvara_model* tvara_model_open_ex(const char* utf8_path, size_t max_blocks, size_t block_tokens,
                                           const tvara_open_options* options);

/* The tensor-parallel shard a rank of tvara_model_open_ex holds (no
 * reference counterpart: the reference engine is single-device).  Query
 * heads, KV heads and FFN rows [begin, begin + count) of each layer; Q/K/V and
 * gate/up are split by rows, o_proj and down_proj by the matching columns,
 * and the partial outputs of o_proj / down_proj are summed over the group.
 * Reads only the GGUF header (no GPU).  0, or -1 with the reason when the
 * model cannot be split that way. */
typedef struct tvara_tp_shard_info {
    uint32_t struct_size;  /* sizeof(tvara_tp_shard_info) */
    uint32_t head_dim;
    uint32_t heads_begin, heads;
    uint32_t kv_heads_begin, kv_heads;
    uint32_t ffn_begin, ffn;
} tvara_tp_shard_info;
TVARA_API int tvara_tp_shard(const char* utf8_path, uint32_t tp_rank, uint32_t tp_size, tvara_tp_shard_info* out);

/* Device bytes of the packed weights and of the FP16 weight planes (0 when
 * not built).  0 / -1. */
TVARA_API int tvara_model_weight_bytes(tvara_model* model, size_t* packed, size_t* planes);

/* ---- additive: ragged multi-sequence step ----------------------------- */

enum {
    TVARA_STEP_ALL_LOGITS = 1,   /* one logits row per token instead of per sequence */
    TVARA_STEP_FINITE_ARGMAX = 2 /* argmax is 0xFFFFFFFF for a row whose logits hold a NaN or an
                                    infinity: the "Nonfinite model logits" check of
                                    NativeSchedulerBackend.decode_batch (python/tvara/scheduler.py:205-206)
                                    done on the device, without copying logits to the host */
};

/* One device step over a ragged batch: sequence i appends
 * tokens[cu_tokens[i] .. cu_tokens[i+1]) (cu_tokens has n_seq+1 entries,
 * cu_tokens[0] == 0, each range non-empty, each sequence listed once).
 * Prefill chunks and single decode tokens mix freely; this is the
 * scheduler's iteration (python/tvara/scheduler.py:98-122) as one call.
 * Outputs (either may be NULL):
 *   logits  F32 [rows, vocab], rows = n_seq (last token of each sequence)
 *           or total tokens with TVARA_STEP_ALL_LOGITS; count = rows*vocab
 *   argmax  uint32 [rows], the first index of each row's maximum
 * All-or-nothing: on failure every listed sequence is truncated back to its
 * length at entry.  0 / -1. */
TVARA_API int tvara_batch_step(tvara_model* model, size_t n_seq, const uint64_t* sequences,
                               const uint32_t* cu_tokens, const uint32_t* tokens, uint32_t flags, float* logits,
                               size_t count, uint32_t* argmax, size_t argmax_count);

/* Device-side logit post-processing of a step (the sampler of
 * python/tvara/native.py:301-336 up to its random draw, so that only the
 * chosen token or a few candidates cross to the host instead of the
 * full-vocabulary row).  Per sequence, in float64 with
 * the reference's numpy operations: repetition / frequency / presence
 * penalties from the tokens already in the sequence (this step's included),
 * then the token mask (token_masks.py:228-241: disallowed -> -inf).
 * Arrays are indexed by the step's sequence order; NULL parameters take the
 * neutral values 1, 0, 0 and NULL `allowed` allows every token. */
typedef struct tvara_sampling {
    size_t struct_size;          /* sizeof(tvara_sampling) */
    const double* repetition;    /* [n_seq] > 0, or NULL */
    const double* frequency;     /* [n_seq], or NULL */
    const double* presence;      /* [n_seq], or NULL */
    const uint32_t* allowed;     /* [n_seq][ceil(vocab/32)] bit t%32 of word t/32, or NULL */
    uint32_t top_k;              /* candidates returned per sequence, 0..64 */
} tvara_sampling;

enum {
    TVARA_SAMPLE_NONFINITE_LOGITS = 1,   /* "Nonfinite model logits" (native.py:304-305) */
    TVARA_SAMPLE_NONFINITE_ADJUSTED = 2, /* "Nonfinite adjusted sampling logits" (native.py:312-313) */
    TVARA_SAMPLE_NONE_ALLOWED = 4        /* "No grammar-valid tokens remain" (token_masks.py:237-238) */
};

/* tvara_batch_step (one row per sequence) followed by the post-processing
 * above on the device.  Outputs (host, any may be NULL):
 *   logits     F32 [n_seq][vocab] (count = n_seq*vocab) the rows before
 *              post-processing, as tvara_batch_step returns them
 *   argmax     [n_seq] first index of the maximum of the adjusted, masked
 *              logits (np.argmax)
 *   status     [n_seq] TVARA_SAMPLE_* bits of the reference's checks
 *   top_values [n_seq][top_k] the top_k largest adjusted, masked logits,
 *              value descending, ties by index
 *   top_ids    [n_seq][top_k] their token ids
 * Histories are limited to 16384 tokens.  0 / -1 (all-or-nothing). */
TVARA_API int tvara_batch_sample(tvara_model* model, size_t n_seq, const uint64_t* sequences,
                                 const uint32_t* cu_tokens, const uint32_t* tokens, const tvara_sampling* sampling,
                                 float* logits, size_t count, uint32_t* argmax, int32_t* status,
                                 double* top_values, uint32_t* top_ids);

/* ---- additive: sequence management (core/include/tvara/kv.hpp) -------- */

/* PagedCache::fork (kv.hpp:123-129): a new sequence sharing every block;
 * later appends copy a shared partial tail (copy-on-write).  0 on error. */
TVARA_API uint64_t tvara_sequence_fork(tvara_model* model, uint64_t sequence);
/* Committed length of a sequence.  0 / -1. */
TVARA_API int tvara_sequence_length(tvara_model* model, uint64_t sequence, size_t* length);
/* Pool state: free blocks and capacity.  0 / -1. */
TVARA_API int tvara_kv_stats(tvara_model* model, size_t* available, size_t* max_blocks);
/* PagedCache::audit (kv.hpp:138-146) including prefix-cache references.
 * 0 when the invariants hold, -1 with the violated invariant otherwise. */
TVARA_API int tvara_kv_audit(tvara_model* model);
/* Block table of a sequence: up to capacity (id, generation) pairs; returns
 * the table length through *count.  0 / -1. */
TVARA_API int tvara_sequence_blocks(tvara_model* model, uint64_t sequence, uint64_t* ids, uint64_t* generations,
                                    size_t capacity, size_t* count);
/* Reference count of pool block `id` (BlockPool::references_by_id). */
TVARA_API int tvara_kv_references(tvara_model* model, size_t id, size_t* references);

/* ---- additive: device access ------------------------------------------ */

/* The cudaStream_t all of the handle's device work runs on (steps finish
 * with this stream synchronised).  NULL on error. */
TVARA_API void* tvara_model_stream(tvara_model* model);

/* Device view of the paged KV pool, for KV import (e.g. K/V computed by a
 * separate prefill service) and for benchmarks.  Element (block b, layer l,
 * kind 0=K/1=V, KV head g, slot s, e) lives at
 *   base + ((((b*layers + l)*2 + kind)*kv_heads + g)*block_tokens + s)*head_dim + e
 * in elements of kv_dtype; kv_heads is this handle's share under tensor
 * parallelism. */
typedef struct tvara_kv_pool_info {
    void* base;
    size_t max_blocks;
    size_t block_elements;
    uint32_t kv_dtype;
    uint32_t layers, kv_heads, head_dim, block_tokens;
} tvara_kv_pool_info;
TVARA_API int tvara_kv_pool(tvara_model* model, tvara_kv_pool_info* info);
/* TVARA_KV_I8 pools: the device array of row scales, one F32 per (block,
 * layer, kind, KV head, slot) row -- the row of element offset o is o /
 * head_dim; a row decodes as code * scale.  *scales is NULL for other
 * dtypes.  0 / -1. */
TVARA_API int tvara_kv_pool_scales(tvara_model* model, float** scales);

/* Appends `count` positions to a sequence's block table exactly as decoding
 * would (block allocation, copy-on-write of a shared tail) without computing
 * their K/V; those slots hold whatever the pool holds until written through
 * tvara_kv_pool.  All-or-nothing.  0 / -1. */
TVARA_API int tvara_sequence_reserve(tvara_model* model, uint64_t sequence, size_t count);

/* ---- additive: measurement -------------------------------------------- */

/* Device-time accounting per kernel class: while enabled, each step records
 * CUDA events on the handle's stream around its launch groups.  Enabling
 * resets the totals.  0 / -1. */
TVARA_API int tvara_model_profile(tvara_model* model, int enable);
/* Totals since enabling, in this class order: 0 attention, 1 projections
 * (GEMV/GEMM), 2 final norm + LM head + argmax, 3 other elementwise
 * (embedding, RMSNorm, RoPE/KV write, block copies), 4 collectives, 5 host
 * time with the stream idle between the end of one device step and the first
 * work of the next (caller code included).  Writes up to capacity entries;
 * returns the number of classes, -1 on error. */
TVARA_API int tvara_model_profile_read(tvara_model* model, double* milliseconds, uint64_t* groups, size_t capacity);
/* Kernel launches this library has issued since it was loaded. */
TVARA_API uint64_t tvara_kernel_launches(void);
/* Host->device and device->host bytes the last step on this handle copied
 * (its packed batch description in, its logits/argmax out).  0 / -1. */
TVARA_API int tvara_model_step_bytes(tvara_model* model, uint64_t* h2d, uint64_t* d2h);

/* ---- additive: radix prefix cache (core/include/tvara/radix.hpp) ------ */

/* RadixCache::insert + attach (radix.hpp:41-79): caches `sequence`'s KV
 * under its token path (length must equal token_count); returns the node id,
 * 0 on error. */
TVARA_API uint64_t tvara_prefix_insert(tvara_model* model, const int32_t* tokens, size_t token_count,
                                       uint64_t sequence);
/* RadixCache::reuse (radix.hpp:90-96): a new sequence importing the longest
 * cached prefix of tokens (whole blocks unless partial != 0); the reused
 * length is written to *reused.  0 on error. */
TVARA_API uint64_t tvara_prefix_reuse(tvara_model* model, const int32_t* tokens, size_t token_count, int partial,
                                      size_t* reused);
/* RadixCache::lookup: node and matched token count. */
TVARA_API int tvara_prefix_lookup(tvara_model* model, const int32_t* tokens, size_t token_count, uint64_t* node,
                                  size_t* matched);
/* pin / unpin / touch a node and its ancestors (radix.hpp:99-105). */
TVARA_API int tvara_prefix_pin(tvara_model* model, uint64_t node);
TVARA_API int tvara_prefix_unpin(tvara_model* model, uint64_t node);
TVARA_API int tvara_prefix_touch(tvara_model* model, uint64_t node);
/* RadixCache::evict_one (radix.hpp:113-117): 1 evicted, 0 nothing to evict,
 * -1 error. */
TVARA_API int tvara_prefix_evict_one(tvara_model* model);
/* Number of cached nodes (RadixCache::size). */
TVARA_API size_t tvara_prefix_size(tvara_model* model);

/* ---- additive: host-only KV accounting book --------------------------- */
/* The engine's block accounting (kv.hpp:36-165 semantics) without a model or
 * GPU, so callers and tests can replay operation sequences.  Handles are
 * independent of any model. */
typedef struct tvara_kv_book tvara_kv_book;
TVARA_API tvara_kv_book* tvara_kv_book_new(size_t layers, size_t kv_heads, size_t head_dim, size_t block_tokens,
                                           size_t max_blocks);
TVARA_API void tvara_kv_book_free(tvara_kv_book* book);
TVARA_API uint64_t tvara_kv_book_create(tvara_kv_book* book);
/* Returns 0, -1 on error, -2 when the pool is exhausted (state unchanged). */
TVARA_API int tvara_kv_book_append(tvara_kv_book* book, uint64_t sequence);
TVARA_API int tvara_kv_book_drop(tvara_kv_book* book, uint64_t sequence);
TVARA_API uint64_t tvara_kv_book_fork(tvara_kv_book* book, uint64_t sequence);
TVARA_API int tvara_kv_book_truncate(tvara_kv_book* book, uint64_t sequence, size_t length);
TVARA_API uint64_t tvara_kv_book_import(tvara_kv_book* book, uint64_t sequence, size_t length);
TVARA_API size_t tvara_kv_book_available(tvara_kv_book* book);
TVARA_API size_t tvara_kv_book_references(tvara_kv_book* book, size_t id);
TVARA_API int tvara_kv_book_table(tvara_kv_book* book, uint64_t sequence, uint64_t* ids, uint64_t* generations,
                                  size_t capacity, size_t* count);
TVARA_API int tvara_kv_book_audit(tvara_kv_book* book);

/* Prefix cache over a host-only book (the same trie the engine uses, with
 * radix.hpp:17-130's node ids, splits, pins and LRU eviction), so its
 * accounting can be replayed without a GPU.  Node ids, return codes and
 * errors are those of the tvara_prefix_* calls above. */
TVARA_API uint64_t tvara_kv_book_prefix_insert(tvara_kv_book* book, const int32_t* tokens, size_t token_count);
TVARA_API int tvara_kv_book_prefix_attach(tvara_kv_book* book, uint64_t node, uint64_t sequence);
TVARA_API int tvara_kv_book_prefix_lookup(tvara_kv_book* book, const int32_t* tokens, size_t token_count,
                                          uint64_t* node, size_t* matched);
TVARA_API uint64_t tvara_kv_book_prefix_reuse(tvara_kv_book* book, const int32_t* tokens, size_t token_count,
                                              int partial, size_t* reused);
TVARA_API int tvara_kv_book_prefix_pin(tvara_kv_book* book, uint64_t node);
TVARA_API int tvara_kv_book_prefix_unpin(tvara_kv_book* book, uint64_t node);
TVARA_API int tvara_kv_book_prefix_touch(tvara_kv_book* book, uint64_t node);
TVARA_API int tvara_kv_book_prefix_evict_one(tvara_kv_book* book);
TVARA_API size_t tvara_kv_book_prefix_size(tvara_kv_book* book);

#ifdef __cplusplus
}
#endif
#endif /* TVARA_CAPI_H */
