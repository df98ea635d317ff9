"""One engine step at the benchmarked shape, checked against BatchOracle --
TEST INFRASTRUCTURE ONLY (used by tests/ and by bench.py's parity check; the
engine never imports it).

The scenario is the benchmark's, scaled to a size the CPU oracle finishes in
seconds:

* `requests` sequences share a `prefix`-position prefix through the radix
  prefix cache (tvara_prefix_insert / tvara_prefix_reuse with partial reuse,
  the reference's radix.hpp:90-96), so they hold the prefix's full blocks in
  common and each request's first append copies the shared partial tail block
  on the device (copy-on-write, kv.hpp:97-101);
* each request then holds U(lo, hi) more positions of its own
  (tvara_sequence_reserve);
* the whole KV pool is written from one seeded host array of every KV head
  (each tensor-parallel rank uploads the heads it holds), so the oracle knows
  every position's K and V, including the copied blocks;
* one tvara_batch_step appends one token to most sequences and 2..8 to a few
  (a ragged multi-token step), all rows' logits returned.

The oracle recomputes every appended row from the same weights and pool
contents.  The check is the north-star bound: |got - want| <= 2e-3 + 1e-3 |want|
on every logit, and the argmax equal on every row whose top two oracle logits
are further apart than the error bound.  F16 pools are a lossy format the
reference does not have (its KV is F32): their oracle stores the step's new
K/V rows in F16 as the pool does, and the bound is doubled (F16_ATOL,
F16_RTOL) -- at the 8B widths a synthetic model moves its logits by ~2e-3
under attention arithmetic that holds 5e-5 at kernel level, and by ~1e-2
under the F16 storage itself.
"""

from __future__ import annotations

import numpy as np

from .model import BatchOracle

ATOL, RTOL = 2e-3, 1e-3
F16_ATOL, F16_RTOL = 4e-3, 2e-3


class _DeviceView:
    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def build_step(model, *, seed, requests, prefix, suffix, extra_rows, rank=0, world=1, f16_values=False):
    """Sets up the sequences on `model` (an open tvara_b200 NativeModel) and
    returns the step to run and what the oracle needs.  Every rank of a
    tensor-parallel model calls it with the same arguments."""
    import torch
    rng = np.random.default_rng(seed)
    vocab = model.vocab_size
    info = model.kv_pool()
    L, hk_local, d, tpb, B = info["layers"], info["kv_heads"], info["head_dim"], info["block_tokens"], info["max_blocks"]
    hk = hk_local * world
    prefix_tokens = rng.integers(0, vocab, prefix).tolist()
    own = rng.integers(suffix[0], suffix[1] + 1, requests)
    first = rng.integers(0, vocab, requests)
    step_tokens = [[int(first[i])] for i in range(requests)]
    for i in rng.choice(requests, size=min(extra_rows, requests), replace=False):
        step_tokens[int(i)] += rng.integers(0, vocab, int(rng.integers(1, 8))).tolist()
    # the whole pool, every KV head: [block][layer][K/V][head][slot][dim]
    full = rng.standard_normal((B, L, 2, hk, tpb, d), dtype=np.float32)
    if info["kv_dtype"] == 1:
        full = full.astype(np.float16)
    elif f16_values:  # F32 pool holding F16-representable values (to compare the two pool types)
        full = full.astype(np.float16).astype(np.float32)
    mine = np.ascontiguousarray(full[:, :, :, rank * hk_local:(rank + 1) * hk_local])
    typestr = "<f2" if info["kv_dtype"] == 1 else "<f4"
    n = B * info["block_elements"]
    assert mine.size == n, (mine.size, n)
    dev = torch.as_tensor(_DeviceView(info["base"], n, typestr), device="cuda")
    dev.copy_(torch.from_numpy(mine.reshape(-1)))
    torch.cuda.synchronize()
    del mine

    src = model._new_sequence()
    model.reserve(src, prefix)
    node = model.prefix_insert(prefix_tokens, src)
    tail = model.sequence_blocks(src)[-1][0] if prefix % tpb else None
    seqs = []
    for i in range(requests):
        s, reused = model.prefix_reuse(prefix_tokens + [int(first[i])], partial=True)
        assert reused == prefix, (reused, prefix)
        model.reserve(s, int(own[i]))
        seqs.append(s)
    model.prefix_pin(node)
    tables = [[b for b, _ in model.sequence_blocks(s)] for s in seqs]
    starts = [prefix + int(own[i]) for i in range(requests)]
    # expected pool: the uploaded values, with each copy-on-write block holding
    # the shared tail it was copied from
    copies = {}
    if tail is not None:
        k = prefix // tpb
        for t in tables:
            assert t[k] != tail
            copies[t[k]] = tail
    return dict(seqs=seqs, tokens=step_tokens, tables=tables, starts=starts, full=full, copies=copies,
                tpb=tpb, layers=L, kv_width=hk * d, src=src, node=node)


def oracle_rows(path, case, max_positions, kv_round=None):
    full, copies, tpb = case["full"], case["copies"], case["tpb"]
    B, L, _, hk, _, d = full.shape

    def history(table, start):
        ids = np.array([copies.get(b, b) for b in table], np.int64)

        def per_layer(layer):
            blocks = full[ids, layer].astype(np.float32)  # [nb, K/V, head, slot, dim]
            kv = blocks.transpose(1, 0, 3, 2, 4).reshape(2, len(ids) * tpb, hk * d)[:, :start]
            return kv[0], kv[1]
        return per_layer

    oracle = BatchOracle(path, max_positions=max_positions)
    batch = [dict(tokens=t, start=s, history=history(tab, s))
             for t, s, tab in zip(case["tokens"], case["starts"], case["tables"])]
    return oracle.step(batch, kv_round)


def compare(got, want, atol=ATOL, rtol=RTOL) -> dict:
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    ok_values = bool(np.all(err <= atol + rtol * np.abs(want)))
    top2 = np.sort(want, axis=1)[:, -2:]
    decisive = (top2[:, 1] - top2[:, 0]) > 2 * (atol + rtol * np.abs(top2[:, 1]))
    same = np.argmax(got, axis=1) == np.argmax(want, axis=1)
    return {"ok": bool(ok_values and np.all(same | ~decisive)), "rows": int(len(want)),
            "max_abs": float(err.max()), "max_rel": float((err / np.maximum(np.abs(want), 1e-30)).max()),
            "argmax_equal": int(same.sum()), "argmax_near_ties": int((~decisive).sum()),
            "bound": f"|d| <= {atol} + {rtol}|want|; argmax equal unless the top two are within 2x that"}
