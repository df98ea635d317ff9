"""Replicated-model serving on the CPU with two gloo ranks.

Each rank takes its share of the requests from shard_requests (no exchange is
needed to agree on it), serves it with its own ContinuousBatcher over a
deterministic toy model, and the outputs are gathered once at the end.  They
must equal a single replica serving every request, and token-at-a-time
greedy decoding of each request: a request's tokens do not depend on which
replica served it or on what it was batched with."""

import socket

import numpy as np


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist
    from tests.test_scheduler import ToyModel
    from tvara_b200.serving import ContinuousBatcher, shard_requests, synthetic_requests

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        reqs = synthetic_requests(40, ToyModel.vocab_size, prompt=(1, 40), output=(1, 16), seed=9)
        mine = [reqs[i] for i in shard_requests(reqs, world)[rank]]
        ContinuousBatcher(ToyModel(), kv_blocks=48, block_tokens=4, prefill_chunk=8, max_step_tokens=32).run(mine)
        got = [None] * world
        dist.all_gather_object(got, {r.key: r.output for r in mine})
        if rank == 0:
            merged = {k: v for part in got for k, v in part.items()}
            np.save(out_path, np.array([merged[r.key] for r in reqs], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_two_replicas_serve_like_one(tmp_path):
    import torch.multiprocessing as mp
    from tests.test_scheduler import ToyModel, serial_greedy
    from tvara_b200.serving import ContinuousBatcher, synthetic_requests

    out = tmp_path / "replicas.npy"
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = list(np.load(out, allow_pickle=True))
    reqs = synthetic_requests(40, ToyModel.vocab_size, prompt=(1, 40), output=(1, 16), seed=9)
    ContinuousBatcher(ToyModel(), kv_blocks=96, block_tokens=4, prefill_chunk=8, max_step_tokens=32).run(reqs)
    assert got == [r.output for r in reqs]
    assert got == [serial_greedy(ToyModel(), r.prompt, r.max_tokens) for r in reqs]
