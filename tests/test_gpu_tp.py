"""Tensor-parallel engine on two GPUs (skipped with fewer): one process per
GPU opens its shard of the tiny model with an NCCL unique id, both ranks run
the same prefill chunk, ragged batch step and decodes in the same order, and
the logits must match the reference's F32 forward (the pinned oracle) within
the logit tolerance on both ranks -- the allreduce leaves every rank with the
same residual, so the ranks' logits are identical.  Both residual allreduces
are covered (peer memory, NCCL), as are the vocabulary-split head's gathered
argmax and the device sampler over the gathered rows."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 2e-3
NEXT = [5, 77, 300, 41]
THEN = [6, 7, 8, 9]


def _rank(rank, world, nccl_id, path, prompts, out, allreduce):
    import os
    import torch
    from tvara_b200.native import NativeModel

    if allreduce == "nccl":
        os.environ["TVARA_ALLREDUCE"] = "nccl"
    torch.cuda.set_device(rank)
    with NativeModel(path, max_blocks=64, block_tokens=16, device=rank, tp_rank=rank, tp_size=world,
                     nccl_id=nccl_id) as m:
        seqs = [m._new_sequence() for _ in prompts]
        # one ragged step: every prompt but its last token, all rows
        chunk, _ = m.batch_step(seqs, [p[:-1] for p in prompts], all_logits=True)
        # then the last tokens one sequence at a time, through the reference ABI call
        last = np.stack([m.logits(s, p[-1]) for s, p in zip(seqs, prompts)])
        # a decode step with the vocabulary-split head's gathered argmax and
        # the device sampler over the reassembled rows
        step, am = m.batch_step(seqs, [[t] for t in NEXT], logits=True, argmax=True, finite_argmax=True)
        smp = m.batch_sample(seqs, [[t] for t in THEN], repetition=1.2, top_k=5, logits=True)
        np.savez(out % rank, chunk=chunk, last=last, step=step, am=am, s_logits=smp["logits"], s_am=smp["argmax"],
                 s_ids=smp["top_ids"])


def _nccl_unique_id():
    import torch  # noqa: F401  (loads the NCCL that torch ships)
    lib = C.CDLL("libnccl.so.2")
    buf = C.create_string_buffer(128)
    assert lib.ncclGetUniqueId(buf) == 0
    return buf.raw


@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
def test_tp2_matches_oracle(tiny_path, tmp_path, allreduce):
    """peer: the residual allreduce runs over NVLink peer memory (the
    default); nccl: NCCL's allreduce (TVARA_ALLREDUCE=nccl)."""
    import torch
    import torch.multiprocessing as mp
    from oracle.model import OracleModel

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(8)
    # the 300-token prompt makes the chunk step's allreduce run on more CTAs
    # than the one-token calls after it (the barrier counts must follow)
    prompts = [rng.integers(0, 512, n).tolist() for n in (9, 3, 17, 300)]
    out = str(tmp_path / "rank%d.npz")
    nccl_id = _nccl_unique_id()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, 2, nccl_id, str(tiny_path), prompts, out, allreduce))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    r0, r1 = np.load(out % 0), np.load(out % 1)
    assert np.array_equal(r0["chunk"], r1["chunk"]) and np.array_equal(r0["last"], r1["last"])
    oracle = OracleModel(tiny_path, max_positions=320)
    refs = [oracle.forward(p) for p in prompts]
    want_chunk = np.concatenate([r[:-1] for r in refs])
    want_last = np.stack([r[-1] for r in refs])
    assert np.abs(r0["chunk"] - want_chunk).max() <= ATOL
    assert np.abs(r0["last"] - want_last).max() <= ATOL
    for k in ("step", "am", "s_logits", "s_am", "s_ids"):
        assert np.array_equal(r0[k], r1[k]), k
    assert np.array_equal(r0["am"], np.argmax(r0["step"], axis=1))
    refs = [oracle.forward(p + [t]) for p, t in zip(prompts, NEXT)]
    assert np.abs(r0["step"] - np.stack([r[-1] for r in refs])).max() <= ATOL
    from oracle import sampler
    hist = [p + [t, u] for p, t, u in zip(prompts, NEXT, THEN)]
    for i in range(len(prompts)):
        adj = sampler.adjust(r0["s_logits"][i], hist[i], 1.2)
        ids, _ = sampler.top_candidates(adj, 5)
        assert r0["s_am"][i] == int(np.argmax(adj)) and r0["s_ids"][i].tolist() == ids.tolist()
