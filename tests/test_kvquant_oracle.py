"""The int8 KV restatement (oracle/kvquant.py) pinned against the reference's
own QuantizedKV.encode (tests/golden/quantized_kv.npz): bit-exact codes and
scales, including zero rows, a scale that underflows to the smallest positive
float, and exact .5 ties (round half to even)."""

import numpy as np
import pytest

from tests.conftest import GOLDEN


def test_encode_reproduces_reference_golden():
    from oracle import kvquant
    g = np.load(GOLDEN / "quantized_kv.npz")
    codes, scales = kvquant.encode(g["rows"])
    assert np.array_equal(codes, g["codes"])
    assert np.array_equal(scales.view(np.uint32), g["scales"].view(np.uint32))
    assert g["scales"][1, 0] == np.nextafter(np.float32(0), np.float32(1))  # the underflow row is covered
    dec = kvquant.decode(codes, scales)
    assert np.array_equal(dec, codes.astype(np.float32) * scales)


def test_encode_rejects_nonfinite():
    from oracle import kvquant
    with pytest.raises(ValueError, match="Nonfinite KV input"):
        kvquant.encode(np.array([[1.0, np.inf]], np.float32))
