"""int8 KV pools (TVARA_KV_I8, the reference's python/tvara/quantized_kv.py
format): the device encode is bit-exact against the reference's own
QuantizedKV.encode; attention over an int8 pool matches the oracle over the
decoded rows; the engine with an int8 pool matches the oracle model whose K/V
pass through the same format."""

import ctypes as C

import numpy as np
import pytest

from tests.conftest import GOLDEN, make_model
from tests.test_gpu_kernels import check, dev, ptr, sync, torch_dev

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def quantize(capi, rows):
    torch = torch_dev()
    n, d = rows.shape
    codes = torch.empty((n, d), dtype=torch.int8, device="cuda")
    scales = torch.empty(n, dtype=torch.float32, device="cuda")
    status = capi.tvara_kv_quantize(ptr(dev(rows.astype(np.float32))), n, d, ptr(codes), ptr(scales), None)
    return status, codes, scales


def test_kv_quantize_bit_exact_reference_golden(capi):
    g = np.load(GOLDEN / "quantized_kv.npz")
    status, codes, scales = quantize(capi, g["rows"])
    check(capi, status)
    sync()
    assert np.array_equal(codes.cpu().numpy(), g["codes"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), g["scales"].ravel().view(np.uint32))


def test_kv_quantize_random_rows_and_nonfinite(capi):
    from oracle import kvquant
    rng = np.random.default_rng(8)
    for d in (16, 64, 128, 256):
        rows = (rng.standard_normal((300, d)) * rng.uniform(1e-6, 1e4, (300, 1))).astype(np.float32)
        status, codes, scales = quantize(capi, rows)
        check(capi, status)
        sync()
        want_c, want_s = kvquant.encode(rows)
        assert np.array_equal(codes.cpu().numpy(), want_c)
        assert np.array_equal(scales.cpu().numpy().view(np.uint32), want_s.ravel().view(np.uint32))
    bad = np.ones((4, 32), np.float32)
    bad[2, 5] = np.nan
    status, _, _ = quantize(capi, bad)
    assert status != 0 and b"Nonfinite KV input" in capi.tvara_last_error()


def _int8_attention_case(capi, rng, dim, group, tpb, lengths, spread=0.0):
    """Ragged rows over an int8 pool: within the F32 kernels' tolerance of the
    oracle over the decoded rows.  Slots past each row's length hold codes
    with huge scales, so reading one would show.  `spread`: each slot's rows
    are scaled by 2^U(-spread, spread), so row scales differ by that many
    octaves."""
    from oracle import kvquant
    from tests.test_gpu_kernels import attn_close
    from tvara_b200._bindings import AttentionArgs
    torch = torch_dev()
    L, H = 2, 2
    B = sum((n + tpb - 1) // tpb for n in lengths) + 4
    heads = H * group
    rows = rng.standard_normal((B, L, 2, H, tpb, dim)).astype(np.float32)
    if spread:  # V rows over 2 * spread octaves, K rows over 4
        rows[:, :, 1] *= np.exp2(rng.uniform(-spread, spread, (B, L, H, tpb, 1))).astype(np.float32)
        rows[:, :, 0] *= np.exp2(rng.uniform(-2, 2, (B, L, H, tpb, 1))).astype(np.float32)
    codes, scales = kvquant.encode(rows)
    scales = scales[..., 0].copy()
    perm = list(rng.permutation(B))
    tables, offsets = [], []
    for n in lengths:
        offsets.append(len(tables))
        ids = [int(perm.pop()) for _ in range((n + tpb - 1) // tpb)]
        tables += ids
        last = ids[-1]
        scales[last, :, :, :, n - (len(ids) - 1) * tpb:] = 1e30  # poison the tail slots
    decoded = kvquant.decode(codes, scales[..., None])
    layer = 1
    q = rng.standard_normal((len(lengths), heads * dim)).astype(np.float32)
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.kv_dtype = 2
    a.heads, a.kv_heads, a.head_dim, a.block_tokens = heads, H, dim, tpb
    a.layers, a.layer = L, layer
    a.max_blocks, a.n_queries = B, len(lengths)
    qd, pd, sd = dev(q), dev(codes), dev(scales)
    out = torch.empty((len(lengths), heads * dim), dtype=torch.float32, device="cuda")
    tab = np.ascontiguousarray(tables, np.int32)
    off = np.ascontiguousarray(offsets, np.uint32)
    vis = np.ascontiguousarray(lengths, np.uint32)
    a.q, a.out, a.pool, a.kv_scales = qd.data_ptr(), out.data_ptr(), pd.data_ptr(), sd.data_ptr()
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    n = capi.tvara_paged_attention_workspace(C.byref(a))
    assert n, capi.tvara_last_error()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_paged_attention(C.byref(a), ptr(ws), n, None))
    sync()
    got = out.cpu().numpy()
    for i, (o, length) in enumerate(zip(offsets, lengths)):
        ids = tables[o:o + (length + tpb - 1) // tpb]
        keys = np.stack([decoded[ids[p // tpb], layer, 0, :, p % tpb] for p in range(length)]).astype(np.float64)
        vals = np.stack([decoded[ids[p // tpb], layer, 1, :, p % tpb] for p in range(length)]).astype(np.float64)
        q64 = q[i].astype(np.float64).reshape(heads, dim)
        want = np.empty(heads * dim)
        mag = np.empty(heads * dim)  # weighted mean of |v|: the size of the summands
        for h in range(heads):
            s = keys[:, h // group] @ q64[h] / np.sqrt(dim)
            w = np.exp(s - s.max())
            want[h * dim:(h + 1) * dim] = (w @ vals[:, h // group]) / w.sum()
            mag[h * dim:(h + 1) * dim] = (w @ np.abs(vals[:, h // group])) / w.sum()
        if spread:
            # summands of very different sizes cancel: F32 rounding is relative to them
            assert np.all(np.abs(got[i] - want) <= 2e-5 * (1 + np.abs(want) + mag)), (i, np.abs(got[i] - want).max())
        else:
            assert attn_close(got[i], want), (i, np.abs(got[i] - want).max())


@pytest.mark.parametrize("dim", [32, 64, 128])
@pytest.mark.parametrize("group", [1, 4])
def test_attention_over_int8_pool_matches_decoded_oracle(capi, dim, group):
    _int8_attention_case(capi, np.random.default_rng(dim + group), dim, group, 16, [1, 15, 16, 17, 33, 70])


@pytest.mark.parametrize("dim,group,tpb", [(128, 4, 16), (128, 8, 32), (64, 2, 16), (64, 4, 32)])
def test_attention_int8_long_contexts_and_spread_scales(capi, dim, group, tpb):
    """Contexts long enough to be split over several work items (partials
    merged afterwards), with row scales spread over 24 octaves: the int8
    tensor-core kernel's running V-scale bound rescales O as larger rows
    arrive."""
    rng = np.random.default_rng(300 + dim + group + tpb)
    _int8_attention_case(capi, rng, dim, group, tpb, [5, 250, 1024, 1500, 3001], spread=12.0)


def test_engine_int8_kv_matches_quantized_oracle(tiny_path):
    """Ragged prefill + decode with an int8 pool against the oracle model whose
    K and V rows pass through the reference's int8 format."""
    from oracle.model import OracleModel
    from tvara_b200.native import NativeModel
    ref = OracleModel(tiny_path, max_positions=256, kv_quant=True)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 512, n).tolist() for n in (7, 20, 1)]
    with NativeModel(tiny_path, max_blocks=32, block_tokens=16, kv_dtype="i8") as m:
        assert m.kv_pool()["kv_dtype"] == 2 and m.kv_pool()["scales"]
        seqs = [m._new_sequence() for _ in prompts]
        states = [ref.new_state() for _ in prompts]
        toks = prompts
        for step in range(4):
            logits, am = m.batch_step(seqs, toks, argmax=True)
            for i, ts in enumerate(toks):
                for t in ts:
                    want = ref.decode(states[i], t)
                err = np.abs(logits[i] - want)
                assert np.all(err <= ATOL) and np.all(err <= RTOL * np.abs(want) + ATOL), (step, i, err.max())
            toks = [[int(a)] for a in am]
        m.kv_audit()
