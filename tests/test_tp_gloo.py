"""Tensor-parallel split on the CPU with two gloo ranks.

Each rank asks the library which heads and FFN rows it holds
(tvara_tp_shard, the same plan the engine loads), runs the reference's decode
math (the pinned numpy oracle's primitives) on that shard only, and sums the
o_proj / down_proj partials with a gloo all_reduce -- the exchange the engine
does with NCCL after the same two projections.  The result must equal the
unsharded oracle forward: this pins the shard plan and the reduction points
without a GPU."""

import socket

import numpy as np
import pytest

from tests.conftest import make_model


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mv(w, x):
    # Matrix::multiply's double accumulation (the oracle's matvec caches by
    # object identity, which shard views do not have)
    return (w.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)


def _tp_forward(oracle, shard, tokens, allreduce):
    d = shard["head_dim"]
    h0, H = shard["heads_begin"], shard["heads"]
    g0, G = shard["kv_heads_begin"], shard["kv_heads"]
    f0, F = shard["ffn_begin"], shard["ffn"]
    q_rows = slice(h0 * d, (h0 + H) * d)
    kv_rows = slice(g0 * d, (g0 + G) * d)
    keys = [[] for _ in range(oracle.layers)]
    values = [[] for _ in range(oracle.layers)]
    out = []
    for pos, token in enumerate(tokens):
        x = oracle.embedding[token].astype(np.float32).copy()
        for i, b in enumerate(oracle.blocks):
            xn = oracle.rms_norm(x, b["attn_norm"])
            q = oracle.rotary(_mv(b["attn_q"][q_rows], xn), H, pos)
            k = oracle.rotary(_mv(b["attn_k"][kv_rows], xn), G, pos)
            v = _mv(b["attn_v"][kv_rows], xn)
            keys[i].append(k)
            values[i].append(v)
            k64 = np.array(keys[i], np.float64).reshape(-1, G, d)
            v64 = np.array(values[i], np.float64).reshape(-1, G, d)
            q64 = q.astype(np.float64).reshape(H, d)
            att = np.empty(H * d, np.float32)
            for h in range(H):
                kh = h // (H // G)
                s = k64[:, kh, :] @ q64[h] / np.sqrt(np.float64(d))
                w = np.exp(s - s.max())
                att[h * d:(h + 1) * d] = (w @ v64[:, kh, :]) / w.sum()
            part = b["attn_output"][:, q_rows].astype(np.float64) @ att.astype(np.float64)
            x = (x + allreduce(part)).astype(np.float32)
            xn = oracle.rms_norm(x, b["ffn_norm"])
            ff = oracle.swiglu(_mv(b["ffn_gate"][f0:f0 + F], xn), _mv(b["ffn_up"][f0:f0 + F], xn))
            part = b["ffn_down"][:, f0:f0 + F].astype(np.float64) @ ff.astype(np.float64)
            x = (x + allreduce(part)).astype(np.float32)
        out.append(oracle.matvec(oracle.output, oracle.rms_norm(x, oracle.final_norm)))
    return np.stack(out)


def _rank_main(rank, world, port, path, tokens, out_path):
    import torch
    import torch.distributed as dist
    from oracle.model import OracleModel
    from tvara_b200.native import tp_shard

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        shard = tp_shard(path, rank, world)

        def allreduce(part):
            t = torch.from_numpy(np.ascontiguousarray(part))
            dist.all_reduce(t)
            return t.numpy()

        logits = _tp_forward(OracleModel(path, max_positions=64), shard, tokens, allreduce)
        shards = [None] * world
        dist.all_gather_object(shards, shard)
        if rank == 0:
            np.savez(out_path, logits=logits, shards=np.array([[s[k] for k in sorted(s)] for s in shards]),
                     keys=np.array(sorted(shard)))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_matches_unsharded_oracle(tiny_path, tmp_path):
    import torch.multiprocessing as mp
    from oracle.model import OracleModel

    tokens = [5, 77, 300, 12, 511, 0, 42]
    out = tmp_path / "tp.npz"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tiny_path), tokens, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = np.load(out)
    keys = list(res["keys"])
    shards = [dict(zip(keys, row)) for row in res["shards"]]
    # the two ranks partition every head and FFN row exactly once
    assert [s["heads_begin"] for s in shards] == [0, 4] and all(s["heads"] == 4 for s in shards)
    assert [s["kv_heads_begin"] for s in shards] == [0, 1] and all(s["kv_heads"] == 1 for s in shards)
    assert [s["ffn_begin"] for s in shards] == [0, 344] and all(s["ffn"] == 344 for s in shards)
    ref = OracleModel(tiny_path, max_positions=64).forward(tokens)
    assert np.allclose(res["logits"], ref, atol=1e-4, rtol=1e-5), np.abs(res["logits"] - ref).max()


def test_tp_shard_rejects_uneven_splits(tiny_path, model_dir):
    from tvara_b200 import gguf
    from tvara_b200.native import tp_shard

    assert tp_shard(tiny_path, 0, 1)["heads"] == 8
    for rank, size, msg in [(0, 3, "must divide"), (0, 4, "must divide"), (2, 2, "invalid tensor-parallel rank")]:
        with pytest.raises(RuntimeError, match=msg):
            tp_shard(tiny_path, rank, size)
    # Q4_K columns come in blocks of 256: a split of o_proj's 4 heads x 32 = 128 columns is refused
    cfg = gguf.model_config("tiny", hidden=256, heads=8, kv_heads=8, ffn=512,
                            types={"default": gguf.Q4_K, "ffn_down": gguf.Q4_K})
    path = make_model(model_dir, "q4k_tp", cfg, seed=2)
    assert tp_shard(path, 0, 1)["ffn"] == 512
    with pytest.raises(RuntimeError, match="whole number of blocks"):
        tp_shard(path, 1, 2)
