"""Score patterns that exercise the running softmax reference of the
tensor-core attention kernels (F16 and int8 pools): scores that climb along
the context (the reference moves and O is rescaled every few tiles), scores
that fall (the first tile holds the maximum for good), and a lone spike far
above the rest.  Each against the double-precision oracle over the values the
pool actually holds (F16-rounded, or the int8 rows decoded), within the
attention tests' 5e-5 * (1 + |ref|)."""

import ctypes as C

import numpy as np
import pytest

from tests.test_gpu_kernels import attn_close, check, dev, ptr, sync, torch_dev

pytestmark = pytest.mark.gpu

L, H, D, TPB = 1, 2, 128, 16


def _rows(pattern, lengths, group, rng):
    """Pool rows [B][L][2][H][TPB][D] and per-row block tables for `lengths`,
    with K along each KV head's query direction so the score follows the
    pattern; plus the queries."""
    B = sum((n + TPB - 1) // TPB for n in lengths) + 2
    rows = rng.standard_normal((B, L, 2, H, TPB, D)).astype(np.float32) * 0.3
    dirs = np.sign(rng.standard_normal((H, D))).astype(np.float32)  # |dir|^2 = D
    perm = list(rng.permutation(B))
    tables, offsets = [], []
    for n in lengths:
        offsets.append(len(tables))
        ids = [int(perm.pop()) for _ in range((n + TPB - 1) // TPB)]
        tables += ids
        for p in range(n):
            if pattern == "rising":
                target = 0.1 * p          # score grows by 0.1 per position
            elif pattern == "falling":
                target = 0.1 * (n - p)
            else:                          # spike: one position 40 above the rest
                target = 40.0 if p == n // 3 else 0.0
            b, s = ids[p // TPB], p % TPB
            rows[b, 0, 0, :, s, :] += (target / np.sqrt(D)) * dirs
    heads = H * group
    q = np.repeat(dirs, group, axis=0).reshape(1, heads * D)  # each head along its KV head's direction
    q = np.repeat(q, len(lengths), axis=0) + 0.05 * rng.standard_normal((len(lengths), heads * D))
    return rows, tables, offsets, q.astype(np.float32)


def _oracle(vals, q, tables, offsets, lengths, group):
    heads = H * group
    out = np.empty((len(lengths), heads * D))
    for i, (o, n) in enumerate(zip(offsets, lengths)):
        ids = tables[o:o + (n + TPB - 1) // TPB]
        keys = np.stack([vals[ids[p // TPB], 0, 0, :, p % TPB] for p in range(n)]).astype(np.float64)
        vv = np.stack([vals[ids[p // TPB], 0, 1, :, p % TPB] for p in range(n)]).astype(np.float64)
        q64 = q[i].astype(np.float64).reshape(heads, D)
        for h in range(heads):
            s = keys[:, h // group] @ q64[h] / np.sqrt(D)
            w = np.exp(s - s.max())
            out[i, h * D:(h + 1) * D] = (w @ vv[:, h // group]) / w.sum()
    return out


def _run(capi, pool, scales, kv_dtype, q, tables, offsets, lengths, group):
    from tvara_b200._bindings import AttentionArgs
    torch = torch_dev()
    a = AttentionArgs()
    a.struct_size = C.sizeof(AttentionArgs)
    a.kv_dtype = kv_dtype
    a.heads, a.kv_heads, a.head_dim, a.block_tokens = H * group, H, D, TPB
    a.layers, a.layer = L, 0
    a.max_blocks, a.n_queries = pool.shape[0], len(lengths)
    qd, pd = dev(q), dev(pool)
    sd = dev(scales) if scales is not None else None
    out = torch.empty((len(lengths), H * group * D), dtype=torch.float32, device="cuda")
    tab = np.ascontiguousarray(tables, np.int32)
    off = np.ascontiguousarray(offsets, np.uint32)
    vis = np.ascontiguousarray(lengths, np.uint32)
    a.q, a.out, a.pool = qd.data_ptr(), out.data_ptr(), pd.data_ptr()
    if sd is not None:
        a.kv_scales = sd.data_ptr()
    a.tables, a.tables_len = tab.ctypes.data, len(tab)
    a.table_offset, a.visible = off.ctypes.data, vis.ctypes.data
    n = capi.tvara_paged_attention_workspace(C.byref(a))
    assert n, capi.tvara_last_error()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    check(capi, capi.tvara_paged_attention(C.byref(a), ptr(ws), n, None))
    sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("pattern", ["rising", "falling", "spike"])
@pytest.mark.parametrize("kv", ["f16", "i8"])
@pytest.mark.parametrize("group", [1, 4])
def test_attention_score_trends(capi, pattern, kv, group):
    from oracle import kvquant
    rng = np.random.default_rng({"rising": 1, "falling": 2, "spike": 3}[pattern] * 10 + group)
    lengths = [40, 300, 1000, 2500]
    rows, tables, offsets, q = _rows(pattern, lengths, group, rng)
    if kv == "f16":
        pool = rows.astype(np.float16)
        vals, scales, code = pool.astype(np.float32), None, 1
    else:
        codes, sc = kvquant.encode(rows)
        pool, scales, code = codes, sc[..., 0].copy(), 2
        vals = kvquant.decode(codes, sc)
    got = _run(capi, pool, scales, code, q, tables, offsets, lengths, group)
    want = _oracle(vals, q, tables, offsets, lengths, group)
    for i in range(len(lengths)):
        assert attn_close(got[i], want[i], 5e-5), (i, np.abs(got[i] - want[i]).max())
