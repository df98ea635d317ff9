"""ctypes signatures of every symbol in include/tvara_capi.h and
include/tvara_kernels.h."""

from __future__ import annotations

import ctypes as C

P = C.c_void_p
SZ = C.c_size_t
U64 = C.c_uint64
U32P = C.POINTER(C.c_uint32)
U64P = C.POINTER(C.c_uint64)
I32P = C.POINTER(C.c_int32)
F32P = C.POINTER(C.c_float)
SZP = C.POINTER(C.c_size_t)


class OpenOptions(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("device", C.c_int32),
        ("kv_dtype", C.c_uint32),
        ("max_step_tokens", C.c_uint32),
        ("tp_rank", C.c_uint32),
        ("tp_size", C.c_uint32),
        ("nccl_id", C.c_void_p),
        ("weight_planes", C.c_uint32),
    ]


class TpShardInfo(C.Structure):
    """include/tvara_capi.h tvara_tp_shard_info."""
    _fields_ = [(name, C.c_uint32) for name in (
        "struct_size", "head_dim", "heads_begin", "heads", "kv_heads_begin", "kv_heads", "ffn_begin", "ffn")]


# name: (restype, argtypes)
class Sampling(C.Structure):
    """tvara_sampling: device-side logit post-processing of tvara_batch_sample."""
    _fields_ = [
        ("struct_size", C.c_size_t),
        ("repetition", C.POINTER(C.c_double)),
        ("frequency", C.POINTER(C.c_double)),
        ("presence", C.POINTER(C.c_double)),
        ("allowed", C.POINTER(C.c_uint32)),
        ("top_k", C.c_uint32),
    ]


F64P = C.POINTER(C.c_double)

SIGNATURES = {
    # reference ABI (core/include/tvara/c_api.h:13-24)
    "tvara_model_open": (P, [C.c_char_p, SZ, SZ]),
    "tvara_model_close": (None, [P]),
    "tvara_model_vocab_size": (SZ, [P]),
    "tvara_model_context_size": (SZ, [P]),
    "tvara_last_error": (C.c_char_p, []),
    "tvara_model_metadata": (C.c_char_p, [P]),
    "tvara_sequence_create": (U64, [P]),
    "tvara_sequence_decode": (C.c_int, [P, U64, C.c_uint32, F32P, SZ]),
    "tvara_sequence_drop": (C.c_int, [P, U64]),
    "tvara_sequence_decode_batch": (C.c_int, [P, U64, U32P, SZ, F32P, SZ]),
    "tvara_sequence_truncate": (C.c_int, [P, U64, SZ]),
    # additive
    "tvara_model_open_ex": (P, [C.c_char_p, SZ, SZ, C.POINTER(OpenOptions)]),
    "tvara_model_weight_bytes": (C.c_int, [P, SZP, SZP]),
    "tvara_tp_shard": (C.c_int, [C.c_char_p, C.c_uint32, C.c_uint32, C.POINTER(TpShardInfo)]),
    "tvara_batch_step": (C.c_int, [P, SZ, U64P, U32P, U32P, C.c_uint32, F32P, SZ, U32P, SZ]),
    "tvara_batch_sample": (C.c_int, [P, SZ, U64P, U32P, U32P, C.POINTER(Sampling), F32P, SZ, U32P, I32P, F64P,
                                     U32P]),
    "tvara_kv_pool_scales": (C.c_int, [P, C.POINTER(C.c_void_p)]),
    "tvara_sequence_fork": (U64, [P, U64]),
    "tvara_sequence_length": (C.c_int, [P, U64, SZP]),
    "tvara_kv_stats": (C.c_int, [P, SZP, SZP]),
    "tvara_kv_audit": (C.c_int, [P]),
    "tvara_sequence_blocks": (C.c_int, [P, U64, U64P, U64P, SZ, SZP]),
    "tvara_kv_references": (C.c_int, [P, SZ, SZP]),
    "tvara_model_profile": (C.c_int, [P, C.c_int]),
    "tvara_model_profile_read": (C.c_int, [P, C.POINTER(C.c_double), U64P, SZ]),
    "tvara_kernel_launches": (U64, []),
    "tvara_model_step_bytes": (C.c_int, [P, U64P, U64P]),
    "tvara_model_stream": (P, [P]),
    "tvara_kv_pool": (C.c_int, [P, P]),
    "tvara_sequence_reserve": (C.c_int, [P, U64, SZ]),
    "tvara_prefix_insert": (U64, [P, I32P, SZ, U64]),
    "tvara_prefix_reuse": (U64, [P, I32P, SZ, C.c_int, SZP]),
    "tvara_prefix_lookup": (C.c_int, [P, I32P, SZ, U64P, SZP]),
    "tvara_prefix_pin": (C.c_int, [P, U64]),
    "tvara_prefix_unpin": (C.c_int, [P, U64]),
    "tvara_prefix_touch": (C.c_int, [P, U64]),
    "tvara_prefix_evict_one": (C.c_int, [P]),
    "tvara_prefix_size": (SZ, [P]),
    "tvara_kv_book_new": (P, [SZ, SZ, SZ, SZ, SZ]),
    "tvara_kv_book_free": (None, [P]),
    "tvara_kv_book_create": (U64, [P]),
    "tvara_kv_book_append": (C.c_int, [P, U64]),
    "tvara_kv_book_drop": (C.c_int, [P, U64]),
    "tvara_kv_book_fork": (U64, [P, U64]),
    "tvara_kv_book_truncate": (C.c_int, [P, U64, SZ]),
    "tvara_kv_book_import": (U64, [P, U64, SZ]),
    "tvara_kv_book_available": (SZ, [P]),
    "tvara_kv_book_references": (SZ, [P, SZ]),
    "tvara_kv_book_table": (C.c_int, [P, U64, U64P, U64P, SZ, SZP]),
    "tvara_kv_book_audit": (C.c_int, [P]),
    "tvara_kv_book_prefix_insert": (U64, [P, I32P, SZ]),
    "tvara_kv_book_prefix_attach": (C.c_int, [P, U64, U64]),
    "tvara_kv_book_prefix_lookup": (C.c_int, [P, I32P, SZ, U64P, SZP]),
    "tvara_kv_book_prefix_reuse": (U64, [P, I32P, SZ, C.c_int, SZP]),
    "tvara_kv_book_prefix_pin": (C.c_int, [P, U64]),
    "tvara_kv_book_prefix_unpin": (C.c_int, [P, U64]),
    "tvara_kv_book_prefix_touch": (C.c_int, [P, U64]),
    "tvara_kv_book_prefix_evict_one": (C.c_int, [P]),
    "tvara_kv_book_prefix_size": (SZ, [P]),
    # kernel level (include/tvara_kernels.h)
    "tvara_dequantize": (C.c_int, [C.c_int, P, SZ, P, P]),
    "tvara_packed_bytes": (SZ, [C.c_int, SZ, SZ]),
    "tvara_pack": (C.c_int, [C.c_int, P, SZ, SZ, P, P]),
    "tvara_kv_quantize": (C.c_int, [P, SZ, SZ, P, P, P]),
    "tvara_sample_workspace": (SZ, [SZ, SZ]),
    "tvara_sample_logits": (C.c_int, [P, SZ, SZ, P, U64P, F64P, F64P, F64P, P, C.c_uint32, P, P, P, P, P, SZ,
                                      P]),
    "tvara_quant_matmul_workspace": (SZ, [SZ, SZ]),
    "tvara_quant_matmul": (C.c_int, [C.c_int, P, SZ, SZ, P, SZ, P, P, SZ, P]),
    "tvara_paged_attention_workspace": (SZ, [P]),
    "tvara_paged_attention": (C.c_int, [P, P, SZ, P]),
    "tvara_paged_attention_noalloc_max": (SZ, []),
    "tvara_paged_attention_noalloc": (C.c_int, [P, P]),
}


class AttentionArgs(C.Structure):
    """include/tvara_kernels.h tvara_attention_args."""
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("kv_dtype", C.c_uint32),
        ("heads", C.c_uint32),
        ("kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("block_tokens", C.c_uint32),
        ("layers", C.c_uint32),
        ("layer", C.c_uint32),
        ("max_blocks", C.c_size_t),
        ("n_queries", C.c_size_t),
        ("q", C.c_void_p),
        ("out", C.c_void_p),
        ("pool", C.c_void_p),
        ("tables", C.c_void_p),
        ("tables_len", C.c_size_t),
        ("table_offset", C.c_void_p),
        ("visible", C.c_void_p),
        ("kv_scales", C.c_void_p),
    ]


def declare(lib) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
