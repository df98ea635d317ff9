"""Serving on the GPU engine.

* The reference's own Scheduler (python/tvara/scheduler.py, staged unchanged
  into oracle/_ref/python) over BatchedSchedulerBackend: every iteration is one
  tvara_batch_step.
* The replica serving loop (tvara_b200.serving): requests sharded over two
  engine replicas, each with its own continuous batching of prefill chunks and
  decode tokens.
Every emitted token is the greedy token of the reference's F32 forward (the
pinned numpy oracle) along the request's own history, up to near-ties within
the logit tolerance."""

import numpy as np
import pytest

from oracle import reference_module
from tvara_b200 import gguf
from tvara_b200.native import ARGMAX_NONFINITE, NativeModel
from tvara_b200.scheduler import BatchedSchedulerBackend
from tvara_b200.serving import ContinuousBatcher, shard_requests, synthetic_requests
from tests.conftest import make_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sched():
    mod = reference_module("scheduler")
    if mod is None:
        pytest.skip("reference Python package not staged (oracle/_ref/python)")
    return mod


ATOL = 2e-3


def _check_greedy(oracle, requests):
    exact = total = 0
    for r in requests:
        history = list(r.prompt) + list(r.output)
        if not r.output:
            continue
        logits = oracle.forward(history[:-1])[len(r.prompt) - 1:]
        for row, token in zip(logits, r.output):
            best = float(row.max())
            assert row[token] >= best - 2 * ATOL, (getattr(r, "identifier", None) or r.key, token, best - row[token])
            exact += int(token == int(row.argmax()))
            total += 1
    return exact, total


def test_scheduler_batched_backend_matches_oracle_greedy(sched, tiny_path):
    from oracle.model import OracleModel
    State = sched.State
    oracle = OracleModel(tiny_path, max_positions=512)
    reqs = sched.conversation_load(24, seed=5, vocab=512)
    with NativeModel(tiny_path, max_blocks=96, block_tokens=16) as m:
        backend = BatchedSchedulerBackend(m)
        s = sched.Scheduler(backend, max_active=6, prefill_chunk=3, kv_tokens=256)
        for r in reqs:
            s.submit(r)
        # preempt one request mid-decode and resume it: its replay must not
        # sample anything twice
        for _ in range(6):
            s.step()
        victim = next(r for r in s.active if r.state is State.DECODE)
        s.preempt(victim.identifier)
        s.resume(victim.identifier)
        s.run()
        assert m.kv_stats()[0] == m.kv_stats()[1]  # every block back in the pool
    assert all(r.state is State.FINISHED and len(r.output) == r.max_tokens for r in reqs)
    assert backend.steps < sum(r.max_tokens for r in reqs)  # batched, not serial
    exact, total = _check_greedy(oracle, reqs)
    assert exact == total


def test_replicas_serve_greedy_tokens(tiny_path):
    """Two engine replicas (two handles on one device stand in for two GPUs;
    the sharding and the loop are the same) serve 24 requests with chunked
    prefill; every token is the oracle's greedy token."""
    from oracle.model import OracleModel
    oracle = OracleModel(tiny_path, max_positions=512)
    reqs = synthetic_requests(24, 512, prompt=(1, 70), output=(1, 24), seed=3)
    shards = shard_requests(reqs, 2)
    for part in shards:
        with NativeModel(tiny_path, max_blocks=64, block_tokens=16) as m:
            b = ContinuousBatcher(m, kv_blocks=64, block_tokens=16, prefill_chunk=16, max_step_tokens=48)
            b.run([reqs[i] for i in part])
            assert m.kv_stats()[0] == m.kv_stats()[1]
            assert b.steps < sum(reqs[i].max_tokens + len(reqs[i].prompt) for i in part)
    assert all(len(r.output) == r.max_tokens for r in reqs)
    exact, total = _check_greedy(oracle, reqs)
    assert exact == total


def test_nonfinite_logits_fail_the_iteration(sched, model_dir):
    """An LM-head row of 3e38 overflows the logits (the weights themselves are
    finite, so the model loads, as in the reference)."""
    cfg = gguf.model_config("tiny", tied=False, types={"output": gguf.F32})
    path = model_dir / "overflow.gguf"
    if not path.exists():
        make_model(model_dir, "overflow", cfg, seed=11)
        f = gguf.GGUFFile(path)
        _, shape, off = f.tensors["output.weight"]
        start = f.data_offset + off
        del f
        data = np.memmap(path, dtype=np.uint8, mode="r+")
        row = data[start + 5 * shape[1] * 4:start + 6 * shape[1] * 4].view(np.float32)
        row[:] = 3e38
        data.flush()
        del data, row
    with NativeModel(path, max_blocks=16, block_tokens=16) as m:
        seqs = [m._new_sequence() for _ in range(3)]
        _, plain = m.batch_step(seqs, [[1, 2], [3], [4, 5, 6]], logits=False, argmax=True)
        assert not np.any(plain == ARGMAX_NONFINITE)
        logits, flagged = m.batch_step(seqs, [[7], [8], [9]], logits=True, argmax=True, finite_argmax=True)
        assert not np.isfinite(logits).all(axis=1).any()
        assert np.all(flagged == ARGMAX_NONFINITE)
        for q in seqs:
            m._drop_sequence(q)
        s = sched.Scheduler(BatchedSchedulerBackend(m))
        r = sched.Request("overflow", (1, 2, 3), 2)
        s.submit(r)
        with pytest.raises(ValueError, match="Nonfinite model logits"):
            s.run()
        assert r.state is sched.State.FAILED and not s.active
