"""The scheduler over BatchedSchedulerBackend on the GPU engine: every
iteration is one tvara_batch_step, and every emitted token is the greedy token
of the reference's F32 forward (the pinned numpy oracle) along the request's
own history, up to near-ties within the logit tolerance."""

import numpy as np
import pytest

from tvara_b200 import gguf
from tvara_b200.native import ARGMAX_NONFINITE, NativeModel
from tvara_b200.scheduler import BatchedSchedulerBackend, Request, Scheduler, State, conversation_load
from tests.conftest import make_model

pytestmark = pytest.mark.gpu

ATOL = 2e-3


def _check_greedy(oracle, requests):
    exact = total = 0
    for r in requests:
        history = list(r.prompt) + list(r.output)
        logits = oracle.forward(history[:-1])[len(r.prompt) - 1:]
        for row, token in zip(logits, r.output):
            best = float(row.max())
            assert row[token] >= best - 2 * ATOL, (r.identifier, token, best - row[token])
            exact += int(token == int(row.argmax()))
            total += 1
    return exact, total


def test_scheduler_batched_backend_matches_oracle_greedy(tiny_path):
    from oracle.model import OracleModel
    oracle = OracleModel(tiny_path, max_positions=512)
    reqs = conversation_load(24, seed=5, vocab=512)
    with NativeModel(tiny_path, max_blocks=96, block_tokens=16) as m:
        backend = BatchedSchedulerBackend(m)
        s = Scheduler(backend, max_active=6, prefill_chunk=3, kv_tokens=256)
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


def test_nonfinite_logits_fail_the_iteration(model_dir):
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
        s = Scheduler(BatchedSchedulerBackend(m))
        r = Request("overflow", (1, 2, 3), 2)
        s.submit(r)
        with pytest.raises(ValueError, match="Nonfinite model logits"):
            s.run()
        assert r.state is State.FAILED and not s.active
