"""Scheduler and batched backend on the CPU.

The scheduler cases restate the reference's tests/python/test_scheduler.py
scenarios against tvara_b200.scheduler; when the reference package is
importable, the same seeded workloads are also replayed through the
reference's Scheduler and every backend call is compared.  The batched
backend is checked against a serial backend with the reference's
NativeSchedulerBackend semantics (scheduler.py:186-214) over a deterministic
toy language model, so every emitted token must agree exactly."""

import hashlib
import importlib.util
import random
import sys
from pathlib import Path

import numpy as np
import pytest

from tvara_b200.native import ARGMAX_NONFINITE
from tvara_b200.scheduler import (BatchedSchedulerBackend, Request, Scheduler, State, conversation_load,
                                  latency_report, request_latency)

REFERENCE_SCHEDULER = Path("/root/reference/python/tvara/scheduler.py")


class Recorder:
    """Backend that records every call (tests/python/test_scheduler.py's Backend)."""

    def __init__(self):
        self.live = {}
        self.batches = []
        self.calls = []

    def create(self, key):
        self.calls.append(("create", key))
        self.live[key] = []

    def prefill(self, key, tokens):
        self.calls.append(("prefill", key, tuple(tokens)))
        self.live[key].extend(tokens)

    def decode_batch(self, keys):
        self.calls.append(("decode", tuple(keys)))
        self.batches.append(tuple(keys))
        return [len(self.live[k]) % 7 for k in keys]

    def drop(self, key):
        self.calls.append(("drop", key))
        del self.live[key]


def test_request_validation():
    assert Request("a", (1,), 2).state is State.QUEUED
    for args in [("", (1,), 2), ("a", (), 2), ("a", (-1,), 2), ("a", (1,), -1), ("a", (1.0,), 1)]:
        with pytest.raises(ValueError):
            Request(*args)
    with pytest.raises(ValueError):
        Request("a", (1,), 1, priority=101)


def test_admission_limit_and_duplicate_ids():
    s = Scheduler(Recorder(), 1)
    a = Request("a", (1,), 2)
    s.submit(a)
    s.submit(Request("b", (2,), 1))
    s.admit()
    assert s.active == [a] and len(s.queue) == 1
    with pytest.raises(ValueError):
        s.submit(Request("a", (3,), 1))


def test_one_decode_batch_per_iteration():
    b = Recorder()
    s = Scheduler(b)
    for k in "ab":
        s.submit(Request(k, (1, 2), 2))
    s.step()
    assert b.batches == [("a", "b")] and all(len(r.output) == 1 for r in s.active)


def test_prefill_chunks_and_decode_progress():
    b = Recorder()
    s = Scheduler(b, prefill_chunk=2)
    r = Request("a", (1, 2, 3, 4, 5), 1)
    s.submit(r)
    s.step()
    assert r.position == 2 and not r.output
    s.step()
    assert r.position == 4
    s.step()
    assert r.state is State.FINISHED
    s2 = Scheduler(Recorder(), prefill_chunk=1)
    a, c = Request("a", (1,), 4), Request("c", (1,) * 10, 1)
    s2.submit(a)
    s2.step()
    s2.submit(c)
    s2.step()
    assert len(a.output) == 2 and c.position == 1 and not c.output


def test_kv_budget_priority_aging_pressure():
    s = Scheduler(Recorder(), kv_tokens=4)
    s.submit(Request("a", (1, 2), 2))
    s.submit(Request("b", (1,), 1))
    s.admit()
    assert len(s.active) == 1
    s.run()
    assert all(r.state is State.FINISHED for r in s.requests.values())
    with pytest.raises(ValueError):
        s.submit(Request("c", (1,) * 5, 0))
    s = Scheduler(Recorder(), 1)
    s.submit(Request("low", (1,), 1))
    s.submit(Request("high", (1,), 1, priority=2))
    s.admit()
    assert s.active[0].identifier == "high"
    b = Recorder()
    s = Scheduler(b, kv_tokens=8)
    s.submit(Request("a", (1,), 3))
    s.submit(Request("b", (2,), 3, priority=1))
    s.step()
    s.pressure(4)
    assert s.requests["a"].state is State.PREEMPTED and "a" not in b.live


def test_resume_cancel_and_failures():
    b = Recorder()
    s = Scheduler(b)
    r = Request("a", (1, 2), 3)
    s.submit(r)
    s.step()
    first = list(r.output)
    s.preempt("a")
    s.resume("a")
    s.step()
    assert r.output[:1] == first and len(r.output) == 2
    s.cancel("a")
    assert not b.live and r.state is State.CANCELLED

    class Broken(Recorder):
        def decode_batch(self, keys):
            raise RuntimeError("broken backend")

    b = Broken()
    s = Scheduler(b)
    r = Request("a", (1,), 2)
    s.submit(r)
    with pytest.raises(RuntimeError):
        s.step()
    assert r.state is State.FAILED and not b.live and not s.active


def test_conversation_load_and_latency():
    a, b = conversation_load(), conversation_load()
    assert [(r.prompt, r.max_tokens) for r in a] == [(r.prompt, r.max_tokens) for r in b]
    s = Scheduler(Recorder(), max_active=3, prefill_chunk=2)
    for r in a:
        s.submit(r)
    s.run()
    assert all(len(r.output) == r.max_tokens for r in a)
    r = Request("a", (1,), 3)
    r.submitted, r.token_times, r.output = 1, [2, 2.2, 2.6], [1, 2, 3]
    assert request_latency(r)["ttft_seconds"] == 1
    rep = latency_report([r])
    assert rep["inter_token"]["count"] == 2 and rep["inter_token"]["p50_seconds"] == pytest.approx(0.3)
    assert latency_report([])["ttft"]["p99_seconds"] is None


def _reference_scheduler():
    if not REFERENCE_SCHEDULER.exists():
        return None
    spec = importlib.util.spec_from_file_location("_tvara_reference_scheduler", REFERENCE_SCHEDULER)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def _drive(mod, seed):
    """One seeded session of submits, steps, cancels, preemptions and budget
    changes; returns the backend call trace and the final request states."""
    rng = random.Random(seed)
    b = Recorder()
    s = mod.Scheduler(b, max_active=rng.randint(1, 5), prefill_chunk=rng.randint(1, 4), kv_tokens=64)
    reqs = [mod.Request(r.identifier, r.prompt, r.max_tokens, priority=rng.randint(-3, 3))
            for r in conversation_load(30, seed=seed)]
    pending = list(reqs)
    for it in range(400):
        if pending and rng.random() < 0.5:
            s.submit(pending.pop(0))
        op = rng.random()
        if op < 0.05 and s.active:
            r = rng.choice(s.active)
            if r.state in (mod.State.PREFILL, mod.State.DECODE):
                s.preempt(r.identifier)
                s.resume(r.identifier)
        elif op < 0.08 and s.requests:
            s.cancel(rng.choice(sorted(s.requests)))
        elif op < 0.10:
            s.pressure(rng.randint(24, 64))
        s.step()
        if not pending and not s.active and not s.queue:
            break
    return b.calls, [(r.identifier, r.state.value, tuple(r.output), r.position) for r in reqs]


@pytest.mark.parametrize("seed", range(6))
def test_matches_reference_scheduler_call_for_call(seed):
    ref = _reference_scheduler()
    if ref is None:
        pytest.skip("reference scheduler not present")
    import tvara_b200.scheduler as ours
    assert _drive(ours, seed) == _drive(ref, seed)


# --------------------------------------------------------- batched backend
class ToyModel:
    """Deterministic stand-in for NativeModel: the next-token distribution is
    a function of the sequence's whole token history.  ``logits`` is the
    serial path; ``batch_step`` the batched one."""

    vocab_size = 97

    def __init__(self, poison=None):
        self.history = {}
        self.next_id = 1
        self.poison = poison or set()
        self.steps = []

    def _new_sequence(self):
        self.next_id += 1
        self.history[self.next_id] = []
        return self.next_id

    def _drop_sequence(self, seq):
        del self.history[seq]

    def _row(self, seq):
        h = hashlib.sha256(np.asarray(self.history[seq], np.int64).tobytes()).digest()
        row = np.frombuffer(h * 4, dtype=np.uint8)[:self.vocab_size].astype(np.float32)
        if tuple(self.history[seq]) in self.poison:
            row = row.copy()
            row[3] = np.inf
        return row

    def logits(self, seq, token):
        self.history[seq].append(int(token))
        return self._row(seq)

    def batch_step(self, seqs, token_lists, all_logits=False, logits=True, argmax=False, finite_argmax=False):
        assert not all_logits and argmax and not logits and len(set(seqs)) == len(seqs)
        self.steps.append(sum(len(t) for t in token_lists))
        am = []
        for seq, toks in zip(seqs, token_lists):
            assert len(toks) > 0
            self.history[seq].extend(int(t) for t in toks)
            row = self._row(seq)
            am.append(ARGMAX_NONFINITE if finite_argmax and not np.isfinite(row).all() else int(np.argmax(row)))
        return None, np.asarray(am, np.uint32)


class SerialBackend:
    """NativeSchedulerBackend's behaviour (reference scheduler.py:186-214)."""

    def __init__(self, model):
        self.model, self.sequences, self.pending = model, {}, {}

    def create(self, key):
        self.sequences[key] = self.model._new_sequence()

    def prefill(self, key, tokens):
        for t in tokens:
            self.pending[key] = self.model.logits(self.sequences[key], t)

    def decode_batch(self, keys):
        out = []
        for k in keys:
            row = self.pending[k]
            if not np.isfinite(row).all():
                raise ValueError("Nonfinite model logits")
            t = int(row.argmax())
            out.append(t)
            self.pending[k] = self.model.logits(self.sequences[k], t)
        return out

    def drop(self, key):
        self.model._drop_sequence(self.sequences.pop(key))
        self.pending.pop(key, None)


def _session(backend, seed, preempt=True):
    rng = random.Random(seed)
    s = Scheduler(backend, max_active=rng.randint(2, 6), prefill_chunk=rng.randint(1, 5), kv_tokens=80)
    reqs = conversation_load(24, seed=seed, vocab=ToyModel.vocab_size)
    for r in reqs:
        s.submit(r)
    for _ in range(2000):
        if preempt and s.active and rng.random() < 0.05:
            r = rng.choice(s.active)
            if r.state in (State.PREFILL, State.DECODE):
                s.preempt(r.identifier)
                s.resume(r.identifier)
        s.step()
        s.reap()
        if not s.active and not s.queue:
            break
    return [(r.identifier, r.state, tuple(r.output)) for r in reqs]


@pytest.mark.parametrize("seed", range(5))
def test_batched_backend_emits_serial_tokens(seed):
    serial = _session(SerialBackend(ToyModel()), seed)
    model = ToyModel()
    backend = BatchedSchedulerBackend(model)
    batched = _session(backend, seed)
    assert batched == serial
    assert all(state is State.FINISHED for _, state, _ in batched)
    assert not model.history and not backend.sequences  # every sequence dropped
    # one device step per decoding iteration, prefill chunks folded in
    assert backend.steps == len(model.steps) and sum(model.steps) == backend.step_tokens


def test_batched_backend_nonfinite_fails_iteration():
    reqs = conversation_load(4, seed=3, vocab=ToyModel.vocab_size)
    victim = reqs[2]
    model = ToyModel(poison={victim.prompt})
    s = Scheduler(BatchedSchedulerBackend(model), prefill_chunk=64)
    for r in reqs:
        s.submit(r)
    with pytest.raises(ValueError, match="Nonfinite model logits"):
        s.run()
    assert victim.state is State.FAILED and not s.active and not model.history
    # the serial backend fails the same iteration
    model = ToyModel(poison={victim.prompt})
    s = Scheduler(SerialBackend(model), prefill_chunk=64)
    for r in conversation_load(4, seed=3, vocab=ToyModel.vocab_size):
        s.submit(r)
    with pytest.raises(ValueError, match="Nonfinite model logits"):
        s.run()
