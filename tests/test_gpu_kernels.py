"""Kernel-level parity on the GPU through the C ABI (include/tvara_kernels.h)
against the pinned CPU oracle.

Tolerances: block unpack is bit-exact; projections and attention compute in
F32 against the oracle's double accumulation, so they are checked relative to
the magnitude of the sum: |y - ref| <= 2e-5 * sum|w*x| + 1e-6."""

import ctypes as C

import numpy as np
import pytest

from tvara_b200 import gguf
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

TYPES = (gguf.Q8_0, gguf.Q4_0, gguf.Q4_K, gguf.F16, gguf.F32)


def torch_dev():
    import torch
    return torch


def dev(a):
    torch = torch_dev()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t):
    return C.c_void_p(t.data_ptr())


def sync():
    torch_dev().cuda.synchronize()


def check(lib, status):
    assert status == 0, lib.tvara_last_error().decode()


def test_dequantize_bit_exact_golden(capi):
    g = np.load(GOLDEN / "dequant.npz")
    torch = torch_dev()
    for kind in TYPES:
        raw, want = g[f"raw_{kind}"], g[f"out_{kind}"]
        elems, width = gguf.BLOCK[kind]
        out = torch.empty(want.size, dtype=torch.float32, device="cuda")
        check(capi, capi.tvara_dequantize(kind, ptr(dev(raw)), raw.size // width, ptr(out), None))
        sync()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want), kind


def test_dequantize_bit_exact_random(capi):
    from oracle.oracle import dequantize
    torch = torch_dev()
    rng = np.random.default_rng(5)
    for kind in TYPES:
        elems, width = gguf.BLOCK[kind]
        n = 3000
        raw = rng.integers(0, 256, n * width, dtype=np.uint8)
        out = torch.empty(n * elems, dtype=torch.float32, device="cuda")
        check(capi, capi.tvara_dequantize(kind, ptr(dev(raw)), n, ptr(out), None))
        sync()
        want = dequantize(kind, raw, n * elems)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32)), kind


def packed(capi, kind, raw, rows, cols):
    torch = torch_dev()
    nbytes = capi.tvara_packed_bytes(kind, rows, cols)
    assert nbytes
    buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_pack(kind, ptr(dev(raw)), rows, cols, ptr(buf), None))
    return buf


def matmul(capi, kind, buf, rows, cols, x):
    torch = torch_dev()
    xd = dev(x.astype(np.float32))
    y = torch.full((x.shape[0], rows), float("nan"), dtype=torch.float32, device="cuda")
    n = capi.tvara_quant_matmul_workspace(cols, x.shape[0])
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_quant_matmul(kind, ptr(buf), rows, cols, ptr(xd), x.shape[0], ptr(y), ptr(ws), n, None))
    sync()
    return y.cpu().numpy()


def oracle_matmul(kind, raw, rows, cols, x):
    """Reference product and the error scale of the single-token integer
    path: sum |x||w| (float rounding) plus sum_j |w_j| 2^-22 max|x| over
    x_j's 32-element block (its fixed-point rounding of x)."""
    from oracle.oracle import dequantize
    w = dequantize(kind, raw, rows * cols).reshape(rows, cols).astype(np.float64)
    x64 = x.astype(np.float64)
    blk = np.repeat(np.abs(x64).reshape(x.shape[0], -1, 32).max(axis=2), 32, axis=1)
    return (x64 @ w.T), np.abs(x64) @ np.abs(w.T) + (blk @ np.abs(w.T)) * 2.0 ** -22 / 2e-5


def make_weights(kind, rows, cols, rng):
    if kind in (gguf.F32, gguf.F16):
        return np.frombuffer(gguf.encode(kind, rng.normal(0, 0.05, (rows, cols))), np.uint8).copy()
    return np.frombuffer(gguf.random_blocks(kind, rows, cols, rng), np.uint8).copy()


@pytest.mark.parametrize("kind", TYPES)
@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 5, 9])
def test_quant_matmul_matches_oracle(capi, kind, tokens):
    rng = np.random.default_rng(100 + kind * 10 + tokens)
    rows, cols = 203, 768 if kind != gguf.Q4_K else 1024
    raw = make_weights(kind, rows, cols, rng)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    got = matmul(capi, kind, packed(capi, kind, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(kind, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6)


@pytest.mark.parametrize("kind", [gguf.Q4_K, gguf.Q8_0, gguf.Q4_0])
@pytest.mark.parametrize("rows,cols", [(1, 4096), (203, 1024), (33, 2816), (77, 14336)])
def test_streamed_gemv_matches_oracle(capi, kind, rows, cols):
    """Single-token GEMV on the streamed path (K a multiple of 256): one row,
    a partial last row group, a K tail chunk shorter than the stage (2816 =
    11 x 256) and a wide K; activations spanning 1e-3..30 per element with a
    few large outliers, which the per-unit fixed-point scale must absorb."""
    rng = np.random.default_rng(rows * 7 + cols + kind)
    raw = make_weights(kind, rows, cols, rng)
    x = (rng.standard_normal((1, cols)) * rng.uniform(1e-3, 30, (1, cols))).astype(np.float32)
    x[0, rng.choice(cols, 4, replace=False)] = [1e3, -2e3, 5e-4, 0.0]
    got = matmul(capi, kind, packed(capi, kind, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(kind, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6), np.abs(got - ref).max()


@pytest.mark.parametrize("kind", TYPES)
@pytest.mark.parametrize("tokens", [16, 33, 200, 256, 300, 512])
def test_tensor_core_matmul_matches_oracle(capi, kind, tokens):
    """tcgen05 path: partial weight-row tiles (rows % 128 != 0), partial and
    multiple token tiles, split-K (few row tiles), every weight type."""
    rng = np.random.default_rng(7 * tokens + kind)
    rows, cols = 331, 1024
    raw = make_weights(kind, rows, cols, rng)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 30, (tokens, 1))).astype(np.float32)
    got = matmul(capi, kind, packed(capi, kind, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(kind, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6), np.abs(got - ref).max()


@pytest.mark.parametrize("tokens", [5, 33, 64, 65, 200, 512])
@pytest.mark.parametrize("rows,cols", [(331, 256), (129, 512), (1000, 768)])
def test_narrow_q4k_rows_matches_oracle(capi, tokens, rows, cols):
    """Q4_K rows of one to three blocks (a tensor-parallel shard of o_proj is
    512 wide at 8 ranks): the min-term tile of the tensor-core kernels is
    wider than the row's sub-blocks (the copy fills the rest with zeros), and
    the small-batch kernel runs a single short chunk."""
    rng = np.random.default_rng(tokens * 13 + rows + cols)
    raw = make_weights(gguf.Q4_K, rows, cols, rng)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 30, (tokens, 1))).astype(np.float32)
    got = matmul(capi, gguf.Q4_K, packed(capi, gguf.Q4_K, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(gguf.Q4_K, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6), np.abs(got - ref).max()


@pytest.mark.parametrize("kind", [gguf.Q8_0, gguf.Q4_0])
@pytest.mark.parametrize("tokens", [5, 8, 9, 17, 33, 64, 65, 100, 128, 129])
@pytest.mark.parametrize("rows,cols", [(300, 576), (129, 4096), (77, 2816)])
def test_small_batch_q8_q4_matches_oracle(capi, kind, tokens, rows, cols):
    """Small batches of Q8_0 / Q4_0 rows (5..32 tokens: the mma.sync kernel
    on the packed rows; more: the tensor-core path): token tiles of 8/16/32,
    partial row tiles, K of 18 blocks
    (a short last chunk, no split), 128 blocks (split K) and 88 blocks (a
    short last chunk), activations spanning four orders of magnitude per
    token with a few outliers."""
    rng = np.random.default_rng(tokens * 37 + rows + cols + kind)
    raw = make_weights(kind, rows, cols, rng)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 30, (tokens, 1))).astype(np.float32)
    x[0, rng.choice(cols, 3, replace=False)] = [1e3, -2e3, 0.0]
    got = matmul(capi, kind, packed(capi, kind, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(kind, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6), np.abs(got - ref).max()


@pytest.mark.parametrize("kind", [gguf.Q4_K, gguf.Q8_0, gguf.Q4_0])
def test_quant_matmul_standalone_config_shape(capi, kind):
    """BASELINE standalone config: 11008 x 4096, d/dmin ~ U(0.001, 0.05)."""
    rng = np.random.default_rng(2026)
    rows, cols = 11008, 4096
    raw = np.frombuffer(gguf.random_blocks(kind, rows, cols, rng), np.uint8).copy()
    buf = packed(capi, kind, raw, rows, cols)
    for tokens in (1, 8, 32, 128, 512):
        x = rng.standard_normal((tokens, cols)).astype(np.float32)
        got = matmul(capi, kind, buf, rows, cols, x)
        sel = rng.choice(rows, 256, replace=False)
        from oracle.oracle import dequantize
        elems, width = gguf.BLOCK[kind]
        rb = cols // elems * width
        sub = np.concatenate([raw[r * rb:(r + 1) * rb] for r in sel])
        ref, mag = oracle_matmul(kind, sub, len(sel), cols, x)
        assert np.all(np.abs(got[:, sel] - ref) <= 2e-5 * mag + 1e-6)


# ------------------------------------------------------------------ attention
class Pool:
    """A device KV pool in the engine layout plus host block tables."""

    def __init__(self, layers, kv_heads, dim, tpb, blocks, dtype=np.float32, rng=None):
        self.L, self.H, self.D, self.tpb, self.B = layers, kv_heads, dim, tpb, blocks
        self.dtype = dtype
        self.rng = rng or np.random.default_rng(0)
        self.data = np.full((blocks, layers, 2, kv_heads, tpb, dim), np.nan, dtype=np.float32)
        self.free = list(self.rng.permutation(blocks))

    def sequence(self, length, scale=1.0):
        nb = (length + self.tpb - 1) // self.tpb
        ids = [int(self.free.pop()) for _ in range(nb)]
        for p in range(length):
            b, s = ids[p // self.tpb], p % self.tpb
            self.data[b, :, :, :, s, :] = scale * self.rng.standard_normal((self.L, 2, self.H, self.D))
        return ids

    def device(self):
        return dev(self.data.astype(self.dtype))

    def host_values(self):
        return self.data.astype(self.dtype).astype(np.float32)


def oracle_attention(q, pool, ids, visible, layer, heads):
    vals = pool.host_values()
    D, H, tpb = pool.D, pool.H, pool.tpb
    g = heads // H
    keys = np.stack([vals[ids[p // tpb], layer, 0, :, p % tpb, :] for p in range(visible)]).astype(np.float64)
    vv = np.stack([vals[ids[p // tpb], layer, 1, :, p % tpb, :] for p in range(visible)]).astype(np.float64)
    out = np.empty(heads * D)
    q64 = q.astype(np.float64).reshape(heads, D)
    for h in range(heads):
        s = keys[:, h // g, :] @ q64[h] / np.sqrt(D)
        w = np.exp(s - s.max())
        out[h * D:(h + 1) * D] = (w @ vv[:, h // g, :]) / w.sum()
    return out


def run_attention(capi, pool, layer, heads, queries, tables, offsets, visible, kv_dtype=0):
    from tvara_b200._bindings import AttentionArgs
    torch = torch_dev()
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.kv_dtype = kv_dtype
    a.heads, a.kv_heads, a.head_dim, a.block_tokens = heads, pool.H, pool.D, pool.tpb
    a.layers, a.layer = pool.L, layer
    a.max_blocks, a.n_queries = pool.B, len(visible)
    qd = dev(queries.astype(np.float32))
    out = torch.empty((len(visible), heads * pool.D), dtype=torch.float32, device="cuda")
    pd = pool.device()
    tab = np.ascontiguousarray(tables, np.int32)
    off = np.ascontiguousarray(offsets, np.uint32)
    vis = np.ascontiguousarray(visible, np.uint32)
    a.q, a.out, a.pool = qd.data_ptr(), out.data_ptr(), pd.data_ptr()
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    n = capi.tvara_paged_attention_workspace(C.byref(a))
    assert n, capi.tvara_last_error()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_paged_attention(C.byref(a), ptr(ws), n, None))
    sync()
    return out.cpu().numpy()


def attn_close(got, ref, tol=2e-5):
    return np.all(np.abs(got - ref) <= tol * (1 + np.abs(ref)))


KV_DTYPES = {"f32": (np.float32, 0, 2e-5), "f16": (np.float16, 1, 5e-5)}


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("dim", [32, 64, 128])
@pytest.mark.parametrize("length", [1, 15, 16, 17, 31, 32, 33])
def test_attention_ragged_lengths_nan_poisoned(capi, dim, length, kv):
    """prefill_t174.cpp pattern: unused tail slots hold NaN, freed blocks hold
    junk; neither may reach the output.  F16 pools of head_dim 64/128 run the
    tensor-core kernel, whose value MMA would turn 0 * NaN into NaN."""
    dtype, code, tol = KV_DTYPES[kv]
    rng = np.random.default_rng(length * 7 + dim)
    pool = Pool(1, 2, dim, 16, 8, dtype=dtype, rng=rng)
    junk = pool.sequence(48, scale=100.0)
    pool.free.extend(junk)  # dropped sequence: its blocks keep junk
    ids = pool.sequence(length)
    q = rng.standard_normal(4 * dim).astype(np.float32)
    got = run_attention(capi, pool, 0, 4, q[None], ids, [0], [length], kv_dtype=code)[0]
    assert attn_close(got, oracle_attention(q, pool, ids, length, 0, 4), tol)


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("kv_heads", [1, 2, 4, 8])
def test_attention_gqa_ratios(capi, kv_heads, kv):
    """prefill_t172.cpp: query/KV head ratios 8/4/2/1."""
    dtype, code, tol = KV_DTYPES[kv]
    rng = np.random.default_rng(kv_heads)
    pool = Pool(2, kv_heads, 64, 16, 16, dtype=dtype, rng=rng)
    ids = pool.sequence(67)
    q = rng.standard_normal(8 * 64).astype(np.float32)
    for layer in (0, 1):
        got = run_attention(capi, pool, layer, 8, q[None], ids, [0], [67], kv_dtype=code)[0]
        assert attn_close(got, oracle_attention(q, pool, ids, 67, layer, 8), tol)


@pytest.mark.parametrize("scale", [1e-3, 1.0, 30.0])
def test_attention_f16_tensor_core_scales_and_blocks(capi, scale):
    """Tensor-core path across query magnitudes (the per-head power-of-two
    scaling keeps tiny and large q exact), 32-slot blocks, head_dim 128, odd
    GQA ratios (3, 6), many rows with split-KV."""
    rng = np.random.default_rng(int(scale * 1000) + 5)
    for heads, kv_heads, tpb in ((6, 2, 32), (9, 3, 16), (8, 1, 16)):
        lens = [int(x) for x in rng.integers(1, 700, 12)] + [2049]
        pool = Pool(1, kv_heads, 128, tpb, sum((n + tpb - 1) // tpb for n in lens) + 2, dtype=np.float16, rng=rng)
        tables, offs = [], []
        for n in lens:
            offs.append(len(tables))
            tables += pool.sequence(n, scale=0.7)
        q = (scale * rng.standard_normal((len(lens), heads * 128))).astype(np.float32)
        got = run_attention(capi, pool, 0, heads, q, tables, offs, lens, kv_dtype=1)
        for i, n in enumerate(lens):
            ref = oracle_attention(q[i], pool, tables[offs[i]:offs[i] + (n + tpb - 1) // tpb], n, 0, heads)
            assert attn_close(got[i], ref, 5e-5), (heads, kv_heads, tpb, n)


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_attention_long_contexts_split(capi, kv):
    """prefill_t177.cpp: contexts 1, 127, 1024, 4097, 8192 in one launch
    (long rows are split across CTAs and merged)."""
    rng = np.random.default_rng(9)
    lens = [1, 127, 1024, 4097, 8192]
    pool = Pool(1, 2, 128, 16, sum((n + 15) // 16 for n in lens) + 4, dtype=np.float16 if kv == "f16" else np.float32,
                rng=rng)
    tables, offs = [], []
    for n in lens:
        offs.append(len(tables))
        tables += pool.sequence(n, scale=0.5)
    q = rng.standard_normal((len(lens), 8 * 128)).astype(np.float32)
    got = run_attention(capi, pool, 0, 8, q, tables, offs, lens, kv_dtype=1 if kv == "f16" else 0)
    for i, n in enumerate(lens):
        ref = oracle_attention(q[i], pool, tables[offs[i]:offs[i] + (n + 15) // 16], n, 0, 8)
        assert attn_close(got[i], ref, 5e-5), n


def test_attention_causal_chunk_future_invariant(capi):
    """prefill_t173.cpp: a chunk of query rows at positions start+i sees only
    [0, start+i]; mutating later positions changes nothing."""
    rng = np.random.default_rng(13)
    pool = Pool(1, 1, 32, 7, 20, rng=rng)
    ids = pool.sequence(39)
    q = rng.standard_normal((13, 4 * 32)).astype(np.float32)
    vis = [12 + i for i in range(13)]
    got = run_attention(capi, pool, 0, 4, q, ids, [0] * 13, vis)
    for i in range(13):
        assert attn_close(got[i], oracle_attention(q[i], pool, ids, vis[i], 0, 4))
    pool.data[ids[38 // 7], :, :, :, 38 % 7, :] = 99999.0
    again = run_attention(capi, pool, 0, 4, q, ids, [0] * 13, vis)
    assert np.array_equal(got, again)


def test_attention_block_size_seven_and_many_rows(capi):
    """Odd block size (prefill_t171.cpp uses 7) and a ragged batch of rows."""
    rng = np.random.default_rng(21)
    pool = Pool(3, 3, 64, 7, 40 * 29 + 8, rng=rng)
    lens = [int(x) for x in rng.integers(1, 200, 40)]
    tables, offs = [], []
    for n in lens:
        offs.append(len(tables))
        tables += pool.sequence(n)
    q = rng.standard_normal((len(lens), 9 * 64)).astype(np.float32)
    got = run_attention(capi, pool, 2, 9, q, tables, offs, lens)
    for i, n in enumerate(lens):
        ref = oracle_attention(q[i], pool, tables[offs[i]:offs[i] + (n + 6) // 7], n, 2, 9)
        assert attn_close(got[i], ref)


@pytest.mark.parametrize("kv", ["f16", "f32"])
@pytest.mark.parametrize("dim,heads,kv_heads,tpb", [(128, 32, 8, 16), (128, 16, 2, 32), (64, 8, 8, 16),
                                                    (64, 16, 8, 16), (128, 8, 4, 16), (64, 9, 3, 16),
                                                    (128, 12, 2, 16), (64, 7, 1, 32)])
def test_attention_prefill_chunks(capi, dim, heads, kv_heads, tpb, kv):
    """Chunked prefill (attention.hpp:85-89 fused_prompt_attention): query
    rows at consecutive positions of one sequence, row i seeing
    [0, start + i].  Runs of rows go to the chunk kernels (one K/V read per
    chunk of 4 * floor(16 / G) rows; F16 pools and F32 pools, the latter as
    exact hi + lo F16 pairs); ragged chunk lengths (1..70 rows), contexts to
    3k, unused tail slots, and a few single decode rows in the same launch."""
    dtype, code, tol = KV_DTYPES[kv]
    rng = np.random.default_rng(dim + heads + tpb)
    lens, rows_of = [], []
    for n, r in [(40, 40), (700, 33), (3000, 70), (17, 5), (129, 2), (1, 1), (256, 16), (900, 1), (64, 17)]:
        lens.append(n)
        rows_of.append(r)
    pool = Pool(1, kv_heads, dim, tpb, sum((n + tpb - 1) // tpb for n in lens) + 4, dtype=dtype, rng=rng)
    tables, offs, vis, toff = [], [], [], []
    for n, r in zip(lens, rows_of):
        o = len(tables)
        tables += pool.sequence(n, scale=0.6)
        for i in range(r):
            vis.append(n - r + i + 1)
            toff.append(o)
        offs.append(o)
    q = rng.standard_normal((len(vis), heads * dim)).astype(np.float32)
    got = run_attention(capi, pool, 0, heads, q, tables, toff, vis, kv_dtype=code)
    k = 0
    for s, (n, r) in enumerate(zip(lens, rows_of)):
        ids = tables[offs[s]:offs[s] + (n + tpb - 1) // tpb]
        for i in range(r):
            ref = oracle_attention(q[k], pool, ids, vis[k], 0, heads)
            assert attn_close(got[k], ref, 5e-5), (n, r, i, np.abs(got[k] - ref).max())
            k += 1


def test_attention_chunk_many_short_runs(capi):
    """Speculative-verify shape: many sequences appending 2..8 rows each, so
    the chunk pieces fill the grid; F16, head_dim 128, G = 4."""
    rng = np.random.default_rng(77)
    tpb, dim, heads, kv_heads = 16, 128, 32, 8
    lens = [int(x) for x in rng.integers(20, 1500, 40)]
    rows_of = [int(x) for x in rng.integers(2, 9, 40)]
    pool = Pool(1, kv_heads, dim, tpb, sum((n + tpb - 1) // tpb for n in lens) + 4, dtype=np.float16, rng=rng)
    tables, offs, vis, toff = [], [], [], []
    for n, r in zip(lens, rows_of):
        o = len(tables)
        tables += pool.sequence(n, scale=0.6)
        offs.append(o)
        for i in range(r):
            vis.append(n - r + i + 1)
            toff.append(o)
    q = rng.standard_normal((len(vis), heads * dim)).astype(np.float32)
    got = run_attention(capi, pool, 0, heads, q, tables, toff, vis, kv_dtype=1)
    k = 0
    for s, (n, r) in enumerate(zip(lens, rows_of)):
        ids = tables[offs[s]:offs[s] + (n + tpb - 1) // tpb]
        for i in range(r):
            assert attn_close(got[k], oracle_attention(q[k], pool, ids, vis[k], 0, heads), 5e-5), (n, r, i)
            k += 1


@pytest.mark.parametrize("tokens", [5, 8, 17, 32, 40, 64, 65])
@pytest.mark.parametrize("rows,cols", [(300, 2816), (129, 4096)])
def test_small_batch_q4k_matches_oracle(capi, tokens, rows, cols):
    """Small batches of Q4_K rows (5..64 tokens: the mma.sync kernel on the
    packed rows, split K where the blocks allow; 65 tokens: tensor cores):
    token tiles of 8/16/32/64, partial row tiles, K of 11 blocks (no split)
    and of 16 blocks (split), activations spanning four orders of magnitude
    per token."""
    rng = np.random.default_rng(tokens * 31 + rows + cols)
    raw = make_weights(gguf.Q4_K, rows, cols, rng)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 30, (tokens, 1))).astype(np.float32)
    got = matmul(capi, gguf.Q4_K, packed(capi, gguf.Q4_K, raw, rows, cols), rows, cols, x)
    ref, mag = oracle_matmul(gguf.Q4_K, raw, rows, cols, x)
    assert np.all(np.abs(got - ref) <= 2e-5 * mag + 1e-6), np.abs(got - ref).max()
