"""tvara_paged_attention_noalloc against tvara_paged_attention through the C
ABI: the same attention on the library's static scratch instead of a caller
workspace, for F32, F16 and int8 pools.  This file is collected last so the
entry is exercised both after the other GPU tests and (run on its own) as the
first call in a fresh process.  Both entries run the same kernels on the same
plan, so their outputs must agree bit for bit; the comparison with the oracle
uses the attention tests' tolerance, 2e-5 * (1 + |ref|) (5e-5 for the
tensor-core kernels' rows checked one by one)."""

import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_kernels import Pool, attn_close, check, dev, oracle_attention, ptr, sync

pytestmark = pytest.mark.gpu

LENS = [1, 17, 300, 1024, 4097]


def _args(heads, kv_heads, dim, tpb, layers, layer, blocks, q, out, pd, tab, off, vis, kv_dtype, scales=None):
    from tvara_b200._bindings import AttentionArgs
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.kv_dtype = kv_dtype
    a.heads, a.kv_heads, a.head_dim, a.block_tokens = heads, kv_heads, dim, tpb
    a.layers, a.layer = layers, layer
    a.max_blocks, a.n_queries = blocks, len(vis)
    a.q, a.out, a.pool = q.data_ptr(), out.data_ptr(), pd.data_ptr()
    a.kv_scales = scales.data_ptr() if scales is not None else None
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    return a


def _case(kv, rng):
    """Pool on the device, tables, queries and the oracle's rows for LENS."""
    heads, H, D, tpb, L = 8, 2, 128, 16, 2
    blocks = sum((n + tpb - 1) // tpb for n in LENS) + 4
    if kv == "i8":
        from oracle import kvquant
        rows = (0.5 * rng.standard_normal((blocks, L, 2, H, tpb, D))).astype(np.float32)
        codes, scales = kvquant.encode(rows)
        scales = scales[..., 0].copy()
        decoded = kvquant.decode(codes, scales[..., None])
        perm = list(rng.permutation(blocks))
        tables, offs = [], []
        for n in LENS:
            offs.append(len(tables))
            ids = [int(perm.pop()) for _ in range((n + tpb - 1) // tpb)]
            tables += ids
            scales[ids[-1], :, :, :, n - (len(ids) - 1) * tpb:] = 1e30  # unread tail slots
        pool = Pool(L, H, D, tpb, blocks, rng=rng)
        pool.data[:] = decoded
        pd, sd = dev(codes), dev(scales)
    else:
        pool = Pool(L, H, D, tpb, blocks, dtype=np.float16 if kv == "f16" else np.float32, rng=rng)
        tables, offs = [], []
        for n in LENS:
            offs.append(len(tables))
            tables += pool.sequence(n, scale=0.5)
        pd, sd = pool.device(), None
    q = dev(rng.standard_normal((len(LENS), heads * D)).astype(np.float32))
    want = [oracle_attention(q[i].cpu().numpy(), pool, tables[offs[i]:offs[i] + (n + tpb - 1) // tpb], n, 1, heads)
            for i, n in enumerate(LENS)]
    return dict(heads=heads, H=H, D=D, tpb=tpb, L=L, blocks=blocks, q=q, pd=pd, sd=sd,
                tab=np.ascontiguousarray(tables, np.int32), off=np.ascontiguousarray(offs, np.uint32),
                vis=np.ascontiguousarray(LENS, np.uint32), want=want,
                kv_dtype={"f32": 0, "f16": 1, "i8": 2}[kv])


def _call_args(c, out):
    return _args(c["heads"], c["H"], c["D"], c["tpb"], c["L"], 1, c["blocks"], c["q"], out, c["pd"], c["tab"],
                 c["off"], c["vis"], c["kv_dtype"], c["sd"])


@pytest.mark.parametrize("kv", ["f32", "f16", "i8"])
def test_noalloc_matches_workspace_entry_two_calls(capi, kv):
    import torch
    c = _case(kv, np.random.default_rng(77))
    shape = (len(LENS), c["heads"] * c["D"])
    out_ws = torch.empty(shape, dtype=torch.float32, device="cuda")
    a = _call_args(c, out_ws)
    n = capi.tvara_paged_attention_workspace(C.byref(a))
    assert 0 < n <= capi.tvara_paged_attention_noalloc_max(), capi.tvara_last_error()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_paged_attention(C.byref(a), ptr(ws), n, None))
    sync()
    want = out_ws.cpu().numpy()
    for i in range(len(LENS)):
        assert attn_close(want[i], c["want"][i], 5e-5), LENS[i]

    for _ in range(2):  # two calls in a row on the same static scratch
        out = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
        check(capi, capi.tvara_paged_attention_noalloc(C.byref(_call_args(c, out)), None))
        sync()
        got = out.cpu().numpy()
        assert np.array_equal(got, want)


def test_noalloc_rejects_oversize_scratch(capi):
    import torch
    from tvara_b200._bindings import AttentionArgs
    limit = capi.tvara_paged_attention_noalloc_max()
    tab = np.zeros(limit // 4 + 1024, np.int32)  # block tables alone exceed the scratch
    off = np.zeros(1, np.uint32)
    vis = np.ones(1, np.uint32)
    out = torch.zeros(8 * 64, dtype=torch.float32, device="cuda")
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.heads, a.kv_heads, a.head_dim, a.block_tokens, a.layers, a.layer = 8, 2, 64, 16, 1, 0
    a.max_blocks, a.n_queries = 1, 1
    a.q, a.out, a.pool = out.data_ptr(), out.data_ptr(), out.data_ptr()
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    assert capi.tvara_paged_attention_workspace(C.byref(a)) > limit
    assert capi.tvara_paged_attention_noalloc(C.byref(a), None) == -1
    assert b"exceeds the static maximum" in capi.tvara_last_error()
    sync()
    assert torch.count_nonzero(out).item() == 0  # nothing was launched


def test_noalloc_rejects_bad_block_ids_and_capture(capi):
    """A block id outside the pool is refused on the host before any launch,
    and so is a call on a stream that is being captured into a graph."""
    import torch
    c = _case("f32", np.random.default_rng(5))
    shape = (len(LENS), c["heads"] * c["D"])
    out = torch.zeros(shape, dtype=torch.float32, device="cuda")
    bad = c["tab"].copy()
    bad[int(c["off"][3]) + 2] = c["blocks"]  # one past the pool
    c_bad = dict(c, tab=bad)
    assert capi.tvara_paged_attention_noalloc(C.byref(_call_args(c_bad, out)), None) == -1
    assert b"outside the KV pool" in capi.tvara_last_error()
    sync()
    assert torch.count_nonzero(out).item() == 0
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        rc = capi.tvara_paged_attention_noalloc(C.byref(_call_args(c, out)), C.c_void_p(side.cuda_stream))
    assert rc == -1 and b"captured" in capi.tvara_last_error()
    del graph
    sync()
    assert torch.count_nonzero(out).item() == 0
    # the entry still works after both refusals
    check(capi, capi.tvara_paged_attention_noalloc(C.byref(_call_args(c, out)), None))
    sync()
    got = out.cpu().numpy()
    for i in range(len(LENS)):
        assert attn_close(got[i], c["want"][i], 5e-5), LENS[i]
