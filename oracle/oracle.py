"""ctypes bindings for the oracle libraries (test infrastructure only)."""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_lib = None
_ref = None
_capi = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build():
    """Compile liboracle.so (and _ref/ when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)


def lib():
    global _lib
    if _lib is None:
        path = ORACLE_DIR / "liboracle.so"
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_half_to_float.restype = C.c_float
        L.orc_dequantize.argtypes = [C.c_int, u8p, C.c_size_t, f32p]
        L.orc_q4k_scale_min.argtypes = [u8p, C.c_int, C.POINTER(C.c_uint), C.POINTER(C.c_uint)]
        L.orc_matvec_f32.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p, f32p]
        L.orc_matmul_f32.argtypes = [f32p, C.c_size_t, f32p, C.c_size_t, C.c_size_t, f32p]
        L.orc_matvec_quant.argtypes = [C.c_int, u8p, C.c_size_t, C.c_size_t, f32p, f32p]
        L.orc_rms_norm.argtypes = [f32p, f32p, C.c_size_t, C.c_float, f32p]
        L.orc_rope_table.argtypes = [C.c_size_t, C.c_size_t, C.c_float, f32p, f32p]
        L.orc_rotary.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float, C.c_int]
        L.orc_swiglu.argtypes = [f32p, f32p, C.c_size_t]
        L.orc_paged_attention.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_size_t, f32p, C.c_size_t, C.c_size_t,
                                          C.c_size_t, np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS"),
                                          C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t, f32p]
        L.orc_cache_new.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t]
        L.orc_cache_new.restype = C.c_void_p
        L.orc_cache_free.argtypes = [C.c_void_p]
        for name in ("create",):
            getattr(L, "orc_cache_" + name).argtypes = [C.c_void_p]
            getattr(L, "orc_cache_" + name).restype = C.c_uint64
        L.orc_cache_append.argtypes = [C.c_void_p, C.c_uint64]
        L.orc_cache_drop.argtypes = [C.c_void_p, C.c_uint64]
        L.orc_cache_fork.argtypes = [C.c_void_p, C.c_uint64]
        L.orc_cache_fork.restype = C.c_uint64
        L.orc_cache_truncate.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t]
        L.orc_cache_import.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t]
        L.orc_cache_import.restype = C.c_uint64
        L.orc_cache_available.argtypes = [C.c_void_p]
        L.orc_cache_available.restype = C.c_size_t
        L.orc_cache_references.argtypes = [C.c_void_p, C.c_size_t]
        L.orc_cache_references.restype = C.c_size_t
        L.orc_cache_generation.argtypes = [C.c_void_p, C.c_size_t]
        L.orc_cache_generation.restype = C.c_uint64
        L.orc_cache_length.argtypes = [C.c_void_p, C.c_uint64]
        L.orc_cache_length.restype = C.c_size_t
        L.orc_cache_table.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]
        L.orc_cache_table.restype = C.c_size_t
        L.orc_cache_free_list.argtypes = [C.c_void_p, C.c_void_p]
        L.orc_cache_free_list.restype = C.c_size_t
        L.orc_cache_audit.argtypes = [C.c_void_p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return (ORACLE_DIR / "_ref" / "libtvara_refshim.so").exists()


def ref():
    """The reference's own kernels and cache (None when not built here)."""
    global _ref
    if _ref is None:
        path = ORACLE_DIR / "_ref" / "libtvara_refshim.so"
        if not path.exists():
            return None
        L = C.CDLL(str(path))
        L.ref_error.restype = C.c_char_p
        L.ref_half_to_float.argtypes = [C.c_uint16]
        L.ref_half_to_float.restype = C.c_float
        L.ref_q4k_scale_min.argtypes = [u8p, C.c_size_t, C.POINTER(C.c_uint), C.POINTER(C.c_uint)]
        L.ref_dequantize.argtypes = [C.c_int, u8p, C.c_size_t, f32p, C.c_size_t]
        L.ref_matvec_f32.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p, f32p]
        L.ref_matvec_quant.argtypes = [C.c_int, u8p, C.c_size_t, C.c_size_t, C.c_size_t, f32p, f32p]
        L.ref_matmul_dispatch.argtypes = [C.c_int, u8p, C.c_size_t, C.c_size_t, C.c_size_t, f32p, C.c_size_t,
                                          f32p, C.c_size_t]
        L.ref_matmul_f32_threads.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, f32p, C.c_size_t]
        L.ref_rms_norm.argtypes = [f32p, f32p, C.c_size_t, C.c_float, f32p]
        L.ref_rotary.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float, C.c_int]
        L.ref_cache_new.argtypes = [C.c_size_t] * 5
        L.ref_cache_new.restype = C.c_void_p
        L.ref_cache_free.argtypes = [C.c_void_p]
        L.ref_cache_create.argtypes = [C.c_void_p]
        L.ref_cache_create.restype = C.c_uint64
        L.ref_cache_append.argtypes = [C.c_void_p, C.c_uint64, f32p, f32p]
        L.ref_cache_drop.argtypes = [C.c_void_p, C.c_uint64]
        L.ref_cache_fork.argtypes = [C.c_void_p, C.c_uint64]
        L.ref_cache_fork.restype = C.c_uint64
        L.ref_cache_truncate.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t]
        L.ref_cache_import.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t]
        L.ref_cache_import.restype = C.c_uint64
        L.ref_cache_available.argtypes = [C.c_void_p]
        L.ref_cache_available.restype = C.c_size_t
        L.ref_cache_references.argtypes = [C.c_void_p, C.c_size_t]
        L.ref_cache_references.restype = C.c_size_t
        L.ref_cache_length.argtypes = [C.c_void_p, C.c_uint64]
        L.ref_cache_length.restype = C.c_size_t
        L.ref_cache_table.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]
        L.ref_cache_table.restype = C.c_size_t
        L.ref_cache_audit.argtypes = [C.c_void_p]
        L.ref_cache_block.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t]
        L.ref_cache_block.restype = C.c_void_p
        L.ref_paged_attention.argtypes = [C.c_void_p, C.c_uint64, C.c_size_t, C.c_size_t, f32p, C.c_void_p,
                                          C.c_void_p, C.c_size_t, f32p]
        L.ref_radix_new.argtypes = [C.c_void_p, C.c_char_p]
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        L.ref_radix_insert.argtypes = [C.c_void_p, i32p, C.c_size_t]
        L.ref_radix_insert.restype = C.c_uint64
        L.ref_radix_lookup.argtypes = [C.c_void_p, i32p, C.c_size_t, C.POINTER(C.c_uint64)]
        L.ref_radix_lookup.restype = C.c_size_t
        L.ref_radix_attach.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64]
        L.ref_radix_reuse.argtypes = [C.c_void_p, i32p, C.c_size_t, C.c_int, C.POINTER(C.c_size_t)]
        L.ref_radix_reuse.restype = C.c_uint64
        for name in ("pin", "unpin", "touch"):
            getattr(L, "ref_radix_" + name).argtypes = [C.c_void_p, C.c_uint64]
        L.ref_radix_evict_one.argtypes = [C.c_void_p]
        L.ref_radix_size.argtypes = [C.c_void_p]
        L.ref_radix_size.restype = C.c_size_t
        _ref = L
    return _ref


def reference_module(name: str):
    """A module of the reference's own Python package (python/tvara/<name>.py),
    staged unchanged into oracle/_ref/python by the Makefile; None when it was
    not staged here."""
    import importlib
    import sys
    root = ORACLE_DIR / "_ref" / "python"
    if not (root / "tvara" / f"{name}.py").exists():
        return None
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    return importlib.import_module(f"tvara.{name}")


def ref_capi():
    """The reference engine's C ABI library (None when not built here)."""
    global _capi
    if _capi is None:
        path = ORACLE_DIR / "_ref" / "libtvara_capi.so"
        if not path.exists():
            return None
        _capi = C.CDLL(str(path))
    return _capi


# ------------------------------------------------------------------ conveniences
def dequantize(kind: int, raw: np.ndarray, count: int) -> np.ndarray:
    from tvara_b200.gguf import BLOCK
    elems, width = BLOCK[kind]
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(count, dtype=np.float32)
    if lib().orc_dequantize(kind, raw, count // elems, out):
        raise ValueError("unsupported type")
    return out


def rope_table(positions: int, dim: int, theta: float):
    cos = np.empty((positions, dim // 2), np.float32)
    sin = np.empty((positions, dim // 2), np.float32)
    lib().orc_rope_table(positions, dim, theta, cos, sin)
    return cos, sin


def matvec_quant(kind: int, raw: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    out = np.empty(rows, np.float32)
    if lib().orc_matvec_quant(kind, np.ascontiguousarray(raw, np.uint8), rows, cols,
                              np.ascontiguousarray(x, np.float32), out):
        raise ValueError("invalid quantized matvec")
    return out
