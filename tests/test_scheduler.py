"""Batched scheduler backend and replica serving loop on the CPU.

The reference's own continuous-batching ``Scheduler`` (python/tvara/scheduler.py,
staged unchanged into oracle/_ref/python) drives ``BatchedSchedulerBackend``;
every emitted token must equal what the reference's serial
``NativeSchedulerBackend`` (scheduler.py:186-214) emits over the same
deterministic toy language model.  The replica loop (tvara_b200.serving) is
checked the same way, and its request sharding for 1..8 ranks."""

import hashlib
import random

import numpy as np
import pytest

from oracle import reference_module
from tvara_b200.native import ARGMAX_NONFINITE
from tvara_b200.scheduler import BatchedSchedulerBackend
from tvara_b200.serving import ContinuousBatcher, ServeRequest, shard_requests, synthetic_requests


@pytest.fixture(scope="module")
def ref_sched():
    mod = reference_module("scheduler")
    if mod is None:
        pytest.skip("reference Python package not staged (oracle/_ref/python)")
    return mod


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


def _session(mod, backend, seed, preempt=True):
    rng = random.Random(seed)
    s = mod.Scheduler(backend, max_active=rng.randint(2, 6), prefill_chunk=rng.randint(1, 5), kv_tokens=80)
    reqs = mod.conversation_load(24, seed=seed, vocab=ToyModel.vocab_size)
    for r in reqs:
        s.submit(r)
    for _ in range(2000):
        if preempt and s.active and rng.random() < 0.05:
            r = rng.choice(s.active)
            if r.state in (mod.State.PREFILL, mod.State.DECODE):
                s.preempt(r.identifier)
                s.resume(r.identifier)
        s.step()
        s.reap()
        if not s.active and not s.queue:
            break
    return [(r.identifier, r.state, tuple(r.output)) for r in reqs]


@pytest.mark.parametrize("seed", range(5))
def test_batched_backend_emits_serial_tokens(ref_sched, seed):
    serial = _session(ref_sched, ref_sched.NativeSchedulerBackend(ToyModel()), seed)
    model = ToyModel()
    backend = BatchedSchedulerBackend(model)
    batched = _session(ref_sched, backend, seed)
    assert batched == serial
    assert all(state is ref_sched.State.FINISHED for _, state, _ in batched)
    assert not model.history and not backend.sequences  # every sequence dropped
    # one device step per decoding iteration, prefill chunks folded in
    assert backend.steps == len(model.steps) and sum(model.steps) == backend.step_tokens


def test_batched_backend_nonfinite_fails_iteration(ref_sched):
    reqs = ref_sched.conversation_load(4, seed=3, vocab=ToyModel.vocab_size)
    victim = reqs[2]
    model = ToyModel(poison={victim.prompt})
    s = ref_sched.Scheduler(BatchedSchedulerBackend(model), prefill_chunk=64)
    for r in reqs:
        s.submit(r)
    with pytest.raises(ValueError, match="Nonfinite model logits"):
        s.run()
    assert victim.state is ref_sched.State.FAILED and not s.active and not model.history
    # the serial backend fails the same iteration
    model = ToyModel(poison={victim.prompt})
    s = ref_sched.Scheduler(ref_sched.NativeSchedulerBackend(model), prefill_chunk=64)
    for r in ref_sched.conversation_load(4, seed=3, vocab=ToyModel.vocab_size):
        s.submit(r)
    with pytest.raises(ValueError, match="Nonfinite model logits"):
        s.run()


# ------------------------------------------------------------ replica serving
def serial_greedy(model, prompt, max_tokens):
    """Token-at-a-time greedy decoding through ``logits`` (the serial path)."""
    seq = model._new_sequence()
    for t in prompt:
        row = model.logits(seq, t)
    out = []
    while len(out) < max_tokens:
        out.append(int(np.argmax(row)))
        if len(out) < max_tokens:
            row = model.logits(seq, out[-1])
    model._drop_sequence(seq)
    return out


@pytest.mark.parametrize("chunk,budget,blocks,seed", [(512, 8192, 4096, 0), (3, 7, 64, 1), (5, 64, 40, 2),
                                                      (1, 1, 16, 3)])
def test_continuous_batcher_emits_serial_tokens(chunk, budget, blocks, seed):
    reqs = synthetic_requests(20, ToyModel.vocab_size, prompt=(1, 30), output=(0, 12), seed=seed)
    want = [serial_greedy(ToyModel(), r.prompt, r.max_tokens) for r in reqs]
    model = ToyModel()
    b = ContinuousBatcher(model, kv_blocks=blocks, block_tokens=4, prefill_chunk=chunk, max_step_tokens=budget)
    b.run(reqs)
    assert [r.output for r in reqs] == want
    assert not model.history  # every sequence dropped
    assert max(model.steps) <= budget and b.decode_tokens + sum(1 for r in reqs if r.max_tokens) >= sum(
        r.max_tokens for r in reqs)
    assert b.prefill_tokens == sum(len(r.prompt) for r in reqs)


def test_continuous_batcher_nonfinite_and_capacity():
    reqs = [ServeRequest("a", [1, 2, 3], 4), ServeRequest("b", [4, 5], 3)]
    model = ToyModel(poison={(4, 5)})
    with pytest.raises(ValueError, match="Nonfinite model logits"):
        ContinuousBatcher(model, kv_blocks=64, block_tokens=4).run(reqs)
    assert not model.history
    with pytest.raises(ValueError, match="exceeds the KV pool"):
        ContinuousBatcher(ToyModel(), kv_blocks=1, block_tokens=4).run([ServeRequest("c", [1] * 5, 1)])


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_requests_least_loaded(world):
    reqs = synthetic_requests(256, 97, seed=4)
    shards = shard_requests(reqs, world)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(reqs)))
    loads = [sum(reqs[i].work for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(r.work for r in reqs)
    assert shard_requests(reqs, world) == shards  # every rank computes the same split

