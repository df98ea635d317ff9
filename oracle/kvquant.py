"""Test infrastructure only: a CPU restatement of the reference's
experimental int8 KV format (python/tvara/quantized_kv.py), the checker for
TVARA_KV_I8 pools.  Nothing in the product imports this module.  Pinned
against the reference's own QuantizedKV.encode through
tests/golden/quantized_kv.npz (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np


def encode(rows):
    """quantized_kv.py:21-30: per row (last axis) scale = max|x| / 127 (1 for
    a zero row, the smallest positive float if that underflows), codes
    rint(x / scale) clipped to [-127, 127]."""
    rows = np.asarray(rows, dtype=np.float32)
    if not np.isfinite(rows).all():
        raise ValueError("Nonfinite KV input")
    maximum = np.max(np.abs(rows), axis=-1, keepdims=True)
    scales = np.where(maximum > 0, maximum / np.float32(127), np.float32(1)).astype(np.float32)
    if (scales == 0).any():
        scales = np.maximum(scales, np.nextafter(np.float32(0), np.float32(1)))
    codes = np.clip(np.rint(rows / scales), -127, 127).astype(np.int8)
    return codes, scales


def decode(codes, scales):
    """quantized_kv.py:49-54: codes as float32 times the row scale."""
    return codes.astype(np.float32) * scales


def roundtrip(rows):
    codes, scales = encode(rows)
    return decode(codes, scales)
