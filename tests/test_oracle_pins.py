"""Pins the CPU oracle (oracle/) before anything is checked against it.

* known-answer vectors of the reference's tests/core/test_quant.cpp
  (half conversion :16-22, Q8/Q4/Q4_K blocks :23-67, the 6-bit scale packing
  round trip :39-55, boundaries :134-145) and test_kv.cpp (:7-46);
* bit-equality with the reference itself compiled here (oracle/_ref) on
  random inputs, and with the golden fixtures the reference produced
  (tests/golden/, written by make_golden.py).
"""

import ctypes as C

import numpy as np
import pytest

from tvara_b200 import gguf
from tests.conftest import GOLDEN


def f32bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_half_known_answers(oracle_lib):
    h = oracle_lib.orc_half_to_float
    assert h(0x3C00) == 1.0 and h(0xC000) == -2.0
    assert h(1) == np.ldexp(np.float32(1), -24)
    assert h(0x7BFF) == 65504.0
    assert np.isinf(h(0x7C00)) and np.isnan(h(0x7E00))
    assert np.signbit(h(0x8000))


def half(buf, value, offset=0):
    buf[offset] = value & 255
    buf[offset + 1] = value >> 8


def dq(kind, raw, n):
    from oracle.oracle import dequantize
    return dequantize(kind, np.asarray(raw, np.uint8), n)


def test_q8_q4_known_blocks():
    b = np.zeros(34, np.uint8)
    half(b, 0x3800)
    b[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    assert np.array_equal(dq(gguf.Q8_0, b, 32), 0.5 * (np.arange(32) - 16))
    b = np.zeros(18, np.uint8)
    half(b, 0x3C00)
    i = np.arange(16)
    b[2:] = (i | ((15 - i) << 4)).astype(np.uint8)
    out = dq(gguf.Q4_0, b, 32)
    assert np.array_equal(out[:16], i - 8) and np.array_equal(out[16:], 7 - i)


def test_q4k_scale_packing_round_trip(oracle_lib):
    scales = np.array([[0, 1, 15, 16, 31, 32, 47, 63]])
    mins = np.array([[63, 47, 32, 31, 16, 15, 1, 0]])
    packed = np.ascontiguousarray(gguf.pack_q4k_scales(scales, mins)[0])
    for g in range(8):
        s, m = C.c_uint(), C.c_uint()
        oracle_lib.orc_q4k_scale_min(packed, g, C.byref(s), C.byref(m))
        assert (s.value, m.value) == (scales[0, g], mins[0, g])


def test_q4k_known_block():
    b = np.zeros(144, np.uint8)
    half(b, 0x3800)
    half(b, 0x3400, 2)
    scales, mins = np.arange(1, 9), np.arange(8, 0, -1)
    b[4:16] = gguf.pack_q4k_scales(scales[None], mins[None])[0]
    i = np.arange(128)
    b[16:] = ((i % 16) | ((15 - i % 16) << 4)).astype(np.uint8)
    out = dq(gguf.Q4_K, b, 256)
    for g in range(8):
        q = (15 - np.arange(32) % 16) if g % 2 else (np.arange(32) % 16)
        assert np.allclose(out[g * 32:(g + 1) * 32], 0.5 * scales[g] * q - 0.25 * mins[g], rtol=1e-6)


def test_quant_boundaries():
    b = np.zeros(34, np.uint8)
    assert np.all(dq(gguf.Q8_0, b, 32) == 0)
    half(b, 0x3C00)
    b[2], b[3] = 128, 127
    out = dq(gguf.Q8_0, b, 32)
    assert out[0] == -128 and out[1] == 127
    b = np.zeros(18, np.uint8)
    half(b, 0x3C00)
    b[2] = 0xF0
    out = dq(gguf.Q4_0, b, 32)
    assert out[0] == -8 and out[16] == 7


def test_dequant_matches_reference_golden():
    g = np.load(GOLDEN / "dequant.npz")
    for kind in (gguf.Q8_0, gguf.Q4_0, gguf.Q4_K, gguf.F16, gguf.F32):
        raw, want = g[f"raw_{kind}"], g[f"out_{kind}"]
        got = f32bits(dq(kind, raw, want.size))
        assert np.array_equal(got, want), kind


def test_dequant_bit_exact_vs_reference_random(ref_shim):
    rng = np.random.default_rng(7)
    for kind in (gguf.Q8_0, gguf.Q4_0, gguf.Q4_K, gguf.F16):
        elems, width = gguf.BLOCK[kind]
        raw = rng.integers(0, 256, 500 * width, dtype=np.uint8)
        n = raw.size // width * elems
        ref = np.empty(n, np.float32)
        assert ref_shim.ref_dequantize(kind, raw, raw.size, ref, n) == 0
        assert np.array_equal(f32bits(dq(kind, raw, n)), f32bits(ref))


def test_matvec_quant_matches_reference(ref_shim):
    from oracle.oracle import matvec_quant
    rng = np.random.default_rng(2026)
    for kind, cols in ((gguf.Q8_0, 256), (gguf.Q4_0, 256), (gguf.Q4_K, 512)):
        raw = np.frombuffer(gguf.random_blocks(kind, 12, cols, rng), np.uint8).copy()
        x = rng.uniform(-4, 4, cols).astype(np.float32)
        ref = np.empty(12, np.float32)
        assert ref_shim.ref_matvec_quant(kind, raw, raw.size, 12, cols, x, ref) == 0
        assert np.array_equal(matvec_quant(kind, raw, 12, cols, x), ref)


def test_norm_and_rope_bit_exact(oracle_lib, ref_shim):
    rng = np.random.default_rng(3)
    for n in (8, 256, 4096):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        a, b = np.empty(n, np.float32), np.empty(n, np.float32)
        oracle_lib.orc_rms_norm(x, w, n, 1e-5, a)
        ref_shim.ref_rms_norm(x, w, n, 1e-5, b)
        assert np.array_equal(f32bits(a), f32bits(b))
    for inter in (0, 1):
        for pos in (0, 1, 17, 3500, 8191):
            x = rng.standard_normal(4 * 64).astype(np.float32)
            a, b = x.copy(), x.copy()
            oracle_lib.orc_rotary(a, 4, 64, pos, 500000.0, inter)
            ref_shim.ref_rotary(b, 4, 64, pos, 500000.0, inter)
            assert np.array_equal(f32bits(a), f32bits(b))


def test_rope_split_and_interleaved_equivalent(oracle_lib):
    # tests/core/test_model.cpp:30-37
    x = np.array([1, 2, 3, 4], np.float32)
    oracle_lib.orc_rotary(x, 1, 4, 1, 10000.0, 0)
    y = np.array([1, 3, 2, 4], np.float32)
    oracle_lib.orc_rotary(y, 1, 4, 1, 10000.0, 1)
    assert np.allclose([y[0], y[1], y[2], y[3]], [x[0], x[2], x[1], x[3]], rtol=1e-6)


def test_paged_attention_matches_reference(oracle_lib, ref_shim):
    rng = np.random.default_rng(11)
    layers, kvh, d, tpb, heads = 2, 2, 8, 7, 4
    cache = ref_shim.ref_cache_new(layers, kvh, d, tpb, 32)
    seq = ref_shim.ref_cache_create(cache)
    width = kvh * d
    for _ in range(53):
        k = rng.standard_normal(layers * width).astype(np.float32)
        v = rng.standard_normal(layers * width).astype(np.float32)
        assert ref_shim.ref_cache_append(cache, seq, k, v) == 0
    n = ref_shim.ref_cache_length(cache, seq)
    ids = (C.c_size_t * 64)()
    gens = (C.c_uint64 * 64)()
    nb = ref_shim.ref_cache_table(cache, seq, ids, gens)
    block_elems = layers * 2 * tpb * width
    pool = np.zeros(32 * block_elems, np.float32)
    for i in range(nb):
        p = ref_shim.ref_cache_block(cache, seq, i * tpb)
        pool[ids[i] * block_elems:(ids[i] + 1) * block_elems] = np.ctypeslib.as_array(
            C.cast(p, C.POINTER(C.c_float)), (block_elems,))
    q = rng.standard_normal(heads * d).astype(np.float32)
    table = np.array([ids[i] for i in range(nb)], np.int64)
    for layer in range(layers):
        for visible in (1, 7, 30, 53):
            a, b = np.empty(heads * d, np.float32), np.empty(heads * d, np.float32)
            assert oracle_lib.orc_paged_attention(q, heads, kvh, d, pool, block_elems, tpb, layer, table, n, None,
                                                  None, visible, a) == 0
            assert ref_shim.ref_paged_attention(cache, seq, layer, heads, q, None, None, visible, b) == 0
            assert np.allclose(a, b, rtol=1e-6, atol=1e-7)
    ref_shim.ref_cache_free(cache)


def test_oracle_model_matches_reference_golden(tmp_path):
    from oracle.model import OracleModel
    g = np.load(GOLDEN / "tiny_q8.npz")
    path = gguf.make_llama(tmp_path / "tiny.gguf", "tiny", seed=0)
    m = OracleModel(path, max_positions=256)
    toks = np.concatenate([g["prompt"], g["greedy"]])
    got = m.forward(toks)
    assert np.array_equal(f32bits(got), f32bits(g["logits"]))
    assert m.greedy(g["prompt"], 64) == g["greedy"].tolist()


def test_oracle_model_mixed_types_matches_reference_golden(tmp_path):
    from oracle.model import OracleModel
    from tests.golden.make_golden import MIXED
    g = np.load(GOLDEN / "tiny_mixed.npz")
    path = gguf.make_llama(tmp_path / "mixed.gguf", gguf.model_config("tiny", **MIXED), seed=3)
    got = OracleModel(path, max_positions=64).forward(g["tokens"])
    assert np.array_equal(f32bits(got), f32bits(g["logits"]))


def _replay(book_ops, seed, steps=400):
    """Random create/append/fork/truncate/drop/import sequence applied to
    every accounting implementation in book_ops; returns per-step states."""
    rng = np.random.default_rng(seed)
    live = []
    for _ in range(steps):
        op = rng.choice(["create", "append", "append", "append", "fork", "truncate", "drop", "import"])
        if op == "create" or not live:
            ids = [b["create"]() for b in book_ops]
            assert len(set(ids)) == 1
            live.append(ids[0])
            continue
        s = live[rng.integers(len(live))]
        if op == "append":
            for _ in range(int(rng.integers(1, 6))):
                codes = [b["append"](s) for b in book_ops]
                assert len(set(codes)) == 1, codes
        elif op == "fork":
            ids = [b["fork"](s) for b in book_ops]
            assert len(set(ids)) == 1
            if ids[0]:
                live.append(ids[0])
        elif op == "truncate":
            n = book_ops[0]["length"](s)
            k = int(rng.integers(0, n + 1))
            assert len({b["truncate"](s, k) for b in book_ops}) == 1
        elif op == "drop":
            assert len({b["drop"](s) for b in book_ops}) == 1
            live.remove(s)
        else:
            n = book_ops[0]["length"](s)
            k = int(rng.integers(0, n + 1))
            ids = [b["import"](s, k) for b in book_ops]
            assert len(set(ids)) == 1
            if ids[0]:
                live.append(ids[0])
        states = [b["state"](live) for b in book_ops]
        assert all(st == states[0] for st in states[1:]), op
        assert all(b["audit"]() == 0 for b in book_ops)


def ref_book(R, blocks, tpb):
    c = R.ref_cache_new(1, 1, 4, tpb, blocks)
    x = np.zeros(4, np.float32)

    def state(live):
        tables = {}
        for s in live:
            ids = (C.c_size_t * 4096)()
            gens = (C.c_uint64 * 4096)()
            n = R.ref_cache_table(c, s, ids, gens)
            tables[s] = [(ids[i], gens[i]) for i in range(n)] + [R.ref_cache_length(c, s)]
        return R.ref_cache_available(c), [R.ref_cache_references(c, i) for i in range(blocks)], tables

    return dict(create=lambda: R.ref_cache_create(c), append=lambda s: R.ref_cache_append(c, s, x, x),
                fork=lambda s: R.ref_cache_fork(c, s), truncate=lambda s, n: R.ref_cache_truncate(c, s, n),
                drop=lambda s: R.ref_cache_drop(c, s), length=lambda s: R.ref_cache_length(c, s),
                **{"import": lambda s, n: R.ref_cache_import(c, s, n)}, state=state,
                audit=lambda: R.ref_cache_audit(c))


def orc_book(L, blocks, tpb):
    c = L.orc_cache_new(blocks, tpb, 100000)

    def state(live):
        tables = {}
        for s in live:
            ids = (C.c_size_t * 4096)()
            gens = (C.c_uint64 * 4096)()
            n = L.orc_cache_table(c, s, ids, gens)
            tables[s] = [(ids[i], gens[i]) for i in range(n)] + [L.orc_cache_length(c, s)]
        return L.orc_cache_available(c), [L.orc_cache_references(c, i) for i in range(blocks)], tables

    return dict(create=lambda: L.orc_cache_create(c), append=lambda s: L.orc_cache_append(c, s),
                fork=lambda s: L.orc_cache_fork(c, s), truncate=lambda s, n: L.orc_cache_truncate(c, s, n),
                drop=lambda s: L.orc_cache_drop(c, s), length=lambda s: L.orc_cache_length(c, s),
                **{"import": lambda s, n: L.orc_cache_import(c, s, n)}, state=state,
                audit=lambda: L.orc_cache_audit(c))


@pytest.mark.parametrize("blocks,tpb,seed", [(8, 2, 0), (16, 3, 1), (64, 16, 2), (5, 4, 3)])
def test_kv_accounting_restatement_matches_reference(oracle_lib, ref_shim, blocks, tpb, seed):
    _replay([ref_book(ref_shim, blocks, tpb), orc_book(oracle_lib, blocks, tpb)], seed)


def test_batch_oracle_equals_token_by_token_executor(tiny_path):
    """BatchOracle (float64 matrix products over all rows of a ragged step)
    reproduces OracleModel.decode token by token, bit for bit, on sequences
    with committed history and several new tokens each."""
    from oracle.model import BatchOracle, OracleModel
    o, b = OracleModel(tiny_path, max_positions=128), BatchOracle(tiny_path, max_positions=128)
    rng = np.random.default_rng(0)
    batch, want = [], []
    for n, m in [(10, 1), (0, 3), (5, 2), (33, 4)]:
        st = o.new_state()
        for t in rng.integers(0, 512, n):
            o.decode(st, int(t))
        hist = {layer: (np.array(st["k"][layer], np.float32).reshape(n, o.kv_width),
                        np.array(st["v"][layer], np.float32).reshape(n, o.kv_width)) for layer in range(o.layers)}
        new = rng.integers(0, 512, m).tolist()
        want += [o.decode(st, t) for t in new]
        batch.append(dict(tokens=new, start=n, history=lambda layer, h=hist: h[layer]))
    assert np.array_equal(b.step(batch), np.stack(want))
