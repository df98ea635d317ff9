"""Iteration scheduler and the batched engine backend.

``Scheduler``, ``Request``, ``State``, ``conversation_load``,
``request_latency`` and ``latency_report`` keep the names, arguments, errors
and admission / preemption rules of the reference's python/tvara/scheduler.py
(lines 8-184, 220-257), so code written against it runs unchanged.  The
scheduler is backend-agnostic: it calls ``create``, ``prefill``,
``decode_batch`` and ``drop`` on a duck-typed backend.

``BatchedSchedulerBackend`` replaces the reference's serial
``NativeSchedulerBackend`` (scheduler.py:186-214), which calls
``NativeModel.logits`` once per token per sequence.  Here every scheduler
iteration becomes ONE ``tvara_batch_step``: the prefill chunks queued since
the last step, and the token each decoding sequence emitted last time, run
together on the device, and only the argmax of each sequence's last row comes
back (the finiteness check is done on the device too).  Tokens returned are
the ones the serial backend returns: the argmax of the logits after the
sequence's last fed token.
"""

from __future__ import annotations

import random
import time
from dataclasses import dataclass, field
from enum import Enum


class State(Enum):
    QUEUED = "queued"
    PREFILL = "prefill"
    DECODE = "decode"
    PREEMPTED = "preempted"
    FINISHED = "finished"
    CANCELLED = "cancelled"
    FAILED = "failed"


_TERMINAL = frozenset({State.FINISHED, State.CANCELLED, State.FAILED})


def _is_int(v) -> bool:
    return type(v) is int


@dataclass
class Request:
    identifier: str
    prompt: tuple[int, ...]
    max_tokens: int
    priority: int = 0
    state: State = State.QUEUED
    position: int = 0
    output: list[int] = field(default_factory=list)
    submitted: float = field(default_factory=time.perf_counter)
    token_times: list[float] = field(default_factory=list)
    error: str | None = None

    def __post_init__(self):
        self.prompt = tuple(self.prompt)
        if not _is_int(self.priority) or abs(self.priority) > 100:
            raise ValueError("Invalid priority")
        valid = (bool(self.identifier) and len(self.prompt) > 0
                 and all(_is_int(t) and t >= 0 for t in self.prompt)
                 and _is_int(self.max_tokens) and self.max_tokens >= 0)
        if not valid:
            raise ValueError("Invalid scheduler request")

    @property
    def reservation(self) -> int:
        """KV positions the request may occupy: prompt plus every output token."""
        return len(self.prompt) + self.max_tokens


class Scheduler:
    """Single-owner iteration scheduler (reference scheduler.py:44-184)."""

    def __init__(self, backend, max_active=8, prefill_chunk=64, kv_tokens=4096):
        for value, message in ((max_active, "Invalid active limit"), (prefill_chunk, "Invalid prefill chunk"),
                               (kv_tokens, "Invalid KV token budget")):
            if not _is_int(value) or value < 1:
                raise ValueError(message)
        self.backend = backend
        self.max_active = max_active
        self.prefill_chunk = prefill_chunk
        self.kv_tokens = kv_tokens
        self.iteration = 0
        self.requests: dict[str, Request] = {}
        self.enqueued: dict[str, int] = {}
        self.active: list[Request] = []
        self.queue: list[Request] = []

    # ------------------------------------------------------------ admission
    def submit(self, request):
        if request.identifier in self.requests:
            raise ValueError("Duplicate request ID")
        if request.state is not State.QUEUED:
            raise ValueError("Request already started")
        if request.reservation > self.kv_tokens:
            raise ValueError("Request exceeds KV reservation")
        self.requests[request.identifier] = request
        self.queue.append(request)
        self.enqueued[request.identifier] = self.iteration

    def _rank(self, r):
        # Priority ages by one step every 8 iterations in the queue; ties go
        # to the earliest enqueued.
        waited = (self.iteration - self.enqueued[r.identifier]) // 8
        return -(r.priority + waited), self.enqueued[r.identifier]

    def admit(self):
        self.queue.sort(key=self._rank)
        while self.queue and len(self.active) < self.max_active:
            head = self.queue[0]
            if sum(r.reservation for r in self.active) + head.reservation > self.kv_tokens:
                break
            del self.queue[0]
            if head.state is State.CANCELLED:
                continue
            try:
                self.backend.create(head.identifier)
            except Exception:
                head.state = State.FAILED
                head.error = "Backend admission failed"
                raise
            head.state = State.PREFILL
            self.active.append(head)

    # ------------------------------------------------------------ iteration
    def _step(self):
        self.iteration += 1
        self.reap()
        self.admit()
        for r in self.active:
            if r.state is not State.PREFILL:
                continue
            replay = r.prompt + tuple(r.output)
            stop = min(len(replay), r.position + self.prefill_chunk)
            self.backend.prefill(r.identifier, replay[r.position:stop])
            r.position = stop
            if stop == len(replay):
                r.state = State.DECODE
        decoding = [r for r in self.active if r.state is State.DECODE and len(r.output) < r.max_tokens]
        if decoding:
            tokens = list(self.backend.decode_batch([r.identifier for r in decoding]))
            if len(tokens) != len(decoding) or not all(_is_int(t) and t >= 0 for t in tokens):
                raise ValueError("Invalid backend batch")
            for r, t in zip(decoding, tokens):
                r.output.append(t)
                r.token_times.append(time.perf_counter())
        for r in self.active:
            if len(r.output) >= r.max_tokens:
                r.state = State.FINISHED
        return bool(self.active or self.queue)

    def step(self):
        try:
            return self._step()
        except Exception:
            for r in self.active:
                r.state = State.FAILED
                r.error = "Backend iteration failed"
            self.reap()
            raise

    def reap(self):
        for r in [r for r in self.active if r.state in _TERMINAL]:
            self.backend.drop(r.identifier)
            self.active.remove(r)

    def run(self, max_iterations=100000):
        for _ in range(max_iterations):
            self.step()
            self.reap()
            if not (self.active or self.queue):
                return
        raise RuntimeError("Scheduler iteration budget exhausted")

    # ------------------------------------------------- preemption / control
    def preempt(self, identifier):
        r = self.requests[identifier]
        if r not in self.active or r.state not in (State.PREFILL, State.DECODE):
            raise ValueError("Request is not preemptible")
        self.backend.drop(identifier)
        self.active.remove(r)
        r.state = State.PREEMPTED
        r.position = 0

    def pressure(self, new_budget):
        if not _is_int(new_budget) or new_budget < 1:
            raise ValueError("Invalid KV budget")
        while sum(r.reservation for r in self.active) > new_budget:
            victim = min(self.active, key=lambda r: (r.priority, -self.enqueued[r.identifier]))
            self.preempt(victim.identifier)
        self.kv_tokens = new_budget

    def resume(self, identifier):
        r = self.requests[identifier]
        if r.state is not State.PREEMPTED:
            raise ValueError("Request is not preempted")
        if r.reservation > self.kv_tokens:
            raise ValueError("Insufficient KV reservation")
        # The replay re-feeds prompt + tokens already emitted; none is sampled twice.
        r.state = State.QUEUED
        self.queue.append(r)
        self.enqueued[identifier] = self.iteration

    def cancel(self, identifier):
        r = self.requests[identifier]
        if r.state in _TERMINAL:
            return
        r.state = State.CANCELLED
        if r in self.queue:
            self.queue.remove(r)
        self.reap()


class BatchedSchedulerBackend:
    """Scheduler backend running each iteration as one device step.

    ``model`` is a :class:`tvara_b200.native.NativeModel`.  Work is kept per
    key as tokens not yet run (``feed``) and the token the next decode emits
    (``ready``, the argmax after the last token run).  ``decode_batch`` runs
    every key's feed in one ``batch_step`` (argmax only, finiteness checked on
    the device), emits ``ready`` for the requested keys and queues each
    emitted token to be run by the next step.  Sequence KV therefore trails
    the serial backend by the last emitted token, which is never observable
    through the scheduler protocol.
    """

    def __init__(self, model, check_finite=True):
        from .native import ARGMAX_NONFINITE
        self.model = model
        self.check_finite = check_finite
        self._nonfinite = ARGMAX_NONFINITE
        self.sequences: dict = {}
        self.feed: dict = {}
        self.ready: dict = {}
        self.steps = 0          # device steps issued
        self.step_tokens = 0    # tokens run through them

    def create(self, key):
        self.sequences[key] = self.model._new_sequence()
        self.feed[key] = []
        self.ready[key] = None

    def prefill(self, key, tokens):
        self.feed[key].extend(int(t) for t in tokens)

    def flush(self):
        """Runs every queued token now (one device step)."""
        keys = [k for k, toks in self.feed.items() if toks]
        if not keys:
            return
        _, am = self.model.batch_step([self.sequences[k] for k in keys], [self.feed[k] for k in keys],
                                      logits=False, argmax=True, finite_argmax=self.check_finite)
        self.steps += 1
        self.step_tokens += sum(len(self.feed[k]) for k in keys)
        for k, t in zip(keys, am):
            self.ready[k] = int(t)
            self.feed[k] = []

    def decode_batch(self, keys):
        self.flush()
        out = []
        for k in keys:
            t = self.ready[k]
            if t is None:
                raise ValueError("Sequence has no logits to decode")
            if self.check_finite and t == self._nonfinite:
                raise ValueError("Nonfinite model logits")
            out.append(t)
            self.ready[k] = None
            self.feed[k] = [t]
        return out

    def drop(self, key):
        self.model._drop_sequence(self.sequences.pop(key))
        self.feed.pop(key, None)
        self.ready.pop(key, None)


def conversation_load(count=16, seed=0, vocab=257):
    """Seeded synthetic requests (reference scheduler.py:217-232): prompts of
    1..12 tokens, 1..8 output tokens, drawn from ``random.Random(seed)`` in the
    same order so the same seed gives the same requests."""
    if count < 1 or vocab < 1:
        raise ValueError("Invalid synthetic workload")
    rng = random.Random(seed)
    requests = []
    for i in range(count):
        prompt = tuple(rng.randrange(vocab) for _ in range(rng.randint(1, 12)))
        requests.append(Request(f"conversation-{i}", prompt, rng.randint(1, 8)))
    return requests


def request_latency(request):
    first = request.token_times[0] - request.submitted if request.token_times else None
    return {"ttft_seconds": first, "tokens": len(request.output), "state": request.state.value}


def latency_report(requests):
    import numpy as np

    requests = list(requests)
    ttft = [r.token_times[0] - r.submitted for r in requests if r.token_times]
    gaps = [b - a for r in requests for a, b in zip(r.token_times, r.token_times[1:])]

    def summary(values):
        out = {"count": len(values)}
        for q in (50, 95, 99):
            out[f"p{q}_seconds"] = float(np.percentile(values, q)) if values else None
        return out

    return {"ttft": summary(ttft), "inter_token": summary(gaps)}
