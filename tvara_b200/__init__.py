"""B200 (sm_100a) engine for Tvara's ragged-batch decode/prefill step.

The engine is the shared library ``libtvara_capi.so`` built from ``csrc/`` by
``python -m tvara_b200.build``.  It exports the reference engine's C ABI
(core/include/tvara/c_api.h) unchanged plus additive entry points, so the
reference's own ``tvara.native.NativeModel`` can load it through
``TVARA_LIBRARY``.  ``tvara_b200.native.NativeModel`` mirrors that class for
environments without the reference package and adds the batched step.

There is no CPU fallback: if the library is missing or no CUDA device is
present, loading fails with an error.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "libtvara_capi.so"

_lib = None


def library_path(explicit=None) -> Path:
    if explicit:
        return Path(explicit).resolve()
    if os.environ.get("TVARA_LIBRARY"):
        return Path(os.environ["TVARA_LIBRARY"]).resolve()
    return LIBRARY_PATH


def load_library(explicit=None) -> ctypes.CDLL:
    """Load libtvara_capi.so (raises FileNotFoundError when it was not built)."""
    global _lib
    path = library_path(explicit)
    if explicit is None and _lib is not None:
        return _lib
    if not path.exists():
        raise FileNotFoundError(f"{path} is missing: build it with `python -m tvara_b200.build`")
    lib = ctypes.CDLL(str(path))
    from ._bindings import declare
    declare(lib)
    if explicit is None:
        _lib = lib
    return lib


__all__ = ["load_library", "library_path", "LIBRARY_PATH", "PACKAGE_DIR"]
