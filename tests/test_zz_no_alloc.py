"""tvara_paged_attention_noalloc against tvara_paged_attention through the C
ABI: the same attention on the library's static scratch instead of a caller
workspace.  This file is collected last so the entry is exercised both after
the other GPU tests and (run on its own) as the first call in a fresh process.
Tolerance: the attention tests' 2e-5 * (1 + |ref|); both entries run the same
kernels, so the outputs are expected to agree bit for bit."""

import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_kernels import Pool, attn_close, check, dev, oracle_attention, ptr, sync

pytestmark = pytest.mark.gpu


def _args(pool, layer, heads, q, out, pd, tab, off, vis, kv_dtype):
    from tvara_b200._bindings import AttentionArgs
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.kv_dtype = kv_dtype
    a.heads, a.kv_heads, a.head_dim, a.block_tokens = heads, pool.H, pool.D, pool.tpb
    a.layers, a.layer = pool.L, layer
    a.max_blocks, a.n_queries = pool.B, len(vis)
    a.q, a.out, a.pool = q.data_ptr(), out.data_ptr(), pd.data_ptr()
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    return a


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_noalloc_matches_workspace_entry_two_calls(capi, kv):
    import torch
    rng = np.random.default_rng(77)
    lens = [1, 17, 300, 1024, 4097]
    kv_dtype = 1 if kv == "f16" else 0
    pool = Pool(2, 2, 128, 16, sum((n + 15) // 16 for n in lens) + 4,
                dtype=np.float16 if kv == "f16" else np.float32, rng=rng)
    tables, offs = [], []
    for n in lens:
        offs.append(len(tables))
        tables += pool.sequence(n, scale=0.5)
    heads = 8
    q = dev(rng.standard_normal((len(lens), heads * 128)).astype(np.float32))
    pd = pool.device()
    tab = np.ascontiguousarray(tables, np.int32)
    off = np.ascontiguousarray(offs, np.uint32)
    vis = np.ascontiguousarray(lens, np.uint32)

    out_ws = torch.empty((len(lens), heads * 128), dtype=torch.float32, device="cuda")
    a = _args(pool, 1, heads, q, out_ws, pd, tab, off, vis, kv_dtype)
    n = capi.tvara_paged_attention_workspace(C.byref(a))
    assert 0 < n <= capi.tvara_paged_attention_noalloc_max()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_paged_attention(C.byref(a), ptr(ws), n, None))
    sync()
    want = out_ws.cpu().numpy()

    for _ in range(2):  # two calls in a row on the same static scratch
        out = torch.full((len(lens), heads * 128), float("nan"), dtype=torch.float32, device="cuda")
        b = _args(pool, 1, heads, q, out, pd, tab, off, vis, kv_dtype)
        check(capi, capi.tvara_paged_attention_noalloc(C.byref(b), None))
        sync()
        got = out.cpu().numpy()
        assert attn_close(got, want)
        for i, ln in enumerate(lens):
            ref = oracle_attention(q[i].cpu().numpy(), pool, tables[offs[i]:offs[i] + (ln + 15) // 16], ln, 1, heads)
            assert attn_close(got[i], ref, 5e-5), ln


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
