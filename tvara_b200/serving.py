"""Replicated-model serving: requests sharded across GPUs, one engine per GPU.

Models whose heads do not split evenly over the GPUs (SmolLM2's 9 query /
3 KV heads) or that are too small to gain from tensor parallelism run as
replicas: every GPU holds the whole model and its own KV pool, the requests
are divided between the GPUs once, up front, and each GPU serves its share
with its own continuous-batching loop.  There is no collective in the step.

``shard_requests`` divides the requests least-loaded first: requests are taken
in decreasing order of work (prompt plus output tokens) and each goes to the
GPU with the least work so far (ties to the lower rank; equal-work requests
keep their submission order), so every rank computes the same assignment from
the same list without communicating.

``ContinuousBatcher`` is the per-GPU loop, the iteration rule of the
reference's ``Scheduler._step`` (python/tvara/scheduler.py:98-122) executed as
one ``tvara_batch_step`` per iteration: each iteration feeds every admitted
request either its next prefill chunk (at most ``prefill_chunk`` prompt
tokens) or the token it emitted last, and brings back only each request's
next token (argmax on the device, finiteness checked there).  A request is
admitted when the KV blocks for its prompt plus its whole output fit beside
the requests already running, so a step never runs out of KV blocks.
"""

from __future__ import annotations

import heapq
import time
from dataclasses import dataclass, field


@dataclass
class ServeRequest:
    key: str
    prompt: list
    max_tokens: int
    output: list = field(default_factory=list)
    first_token_s: float | None = None   # seconds from the start of the run to the first output token
    done_s: float | None = None

    @property
    def work(self) -> int:
        return len(self.prompt) + self.max_tokens


def shard_requests(requests, world: int) -> list[list[int]]:
    """Indices of `requests` for each of `world` ranks, least-loaded first."""
    if world < 1:
        raise ValueError("world size must be positive")
    order = sorted(range(len(requests)), key=lambda i: (-requests[i].work, i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + requests[i].work, r))
    return [sorted(s) for s in shards]


class ContinuousBatcher:
    """Continuous batching of `ServeRequest`s on one NativeModel.

    ``max_step_tokens`` bounds the tokens of one device step (decode tokens
    first, then prefill chunks in admission order); ``kv_blocks`` and
    ``block_tokens`` describe the model's KV pool."""

    def __init__(self, model, kv_blocks: int, block_tokens: int = 16, prefill_chunk: int = 512,
                 max_step_tokens: int = 8192, max_active: int | None = None):
        if prefill_chunk < 1 or max_step_tokens < 1:
            raise ValueError("prefill chunk and step budget must be positive")
        self.model = model
        self.kv_blocks = kv_blocks
        self.tpb = block_tokens
        self.prefill_chunk = prefill_chunk
        self.max_step_tokens = max_step_tokens
        self.max_active = max_active
        self.steps = 0
        self.prefill_tokens = 0
        self.decode_tokens = 0

    def _blocks(self, r: ServeRequest) -> int:
        return -(-r.work // self.tpb)

    def run(self, requests) -> list:
        from .native import ARGMAX_NONFINITE
        queue = list(requests)
        for r in queue:
            if not r.prompt or r.max_tokens < 0:
                raise ValueError("Invalid serving request")
            if self._blocks(r) > self.kv_blocks:
                raise ValueError("Request exceeds the KV pool")
        queue.reverse()  # pop() from the end takes the earliest
        active = []      # [request, sequence, prompt tokens fed]
        held = 0
        t0 = time.perf_counter()
        try:
            while queue or active:
                while queue and (self.max_active is None or len(active) < self.max_active) \
                        and held + self._blocks(queue[-1]) <= self.kv_blocks:
                    r = queue.pop()
                    active.append([r, self.model._new_sequence(), 0])
                    held += self._blocks(r)
                if not active:
                    raise RuntimeError("no request fits the KV pool")
                budget = self.max_step_tokens
                seqs, feeds, members = [], [], []
                for entry in active:  # decoding requests: one token each
                    r, seq, fed = entry
                    if fed == len(r.prompt) and budget:
                        seqs.append(seq)
                        feeds.append([r.output[-1]])
                        members.append((entry, False))
                        budget -= 1
                for entry in active:  # then prefill chunks
                    r, seq, fed = entry
                    if fed < len(r.prompt) and budget:
                        take = min(self.prefill_chunk, len(r.prompt) - fed, budget)
                        seqs.append(seq)
                        feeds.append(r.prompt[fed:fed + take])
                        members.append((entry, True))
                        entry[2] = fed + take
                        budget -= take
                _, am = self.model.batch_step(seqs, feeds, logits=False, argmax=True, finite_argmax=True)
                self.steps += 1
                now = time.perf_counter() - t0
                for (entry, prefilling), feed, tok in zip(members, feeds, am):
                    r = entry[0]
                    if prefilling:
                        self.prefill_tokens += len(feed)
                        if entry[2] < len(r.prompt):
                            continue  # more prompt to feed: this row's argmax is not an output
                    else:
                        self.decode_tokens += 1
                    if len(r.output) < r.max_tokens:
                        if int(tok) == ARGMAX_NONFINITE:
                            raise ValueError("Nonfinite model logits")
                        r.output.append(int(tok))
                        if r.first_token_s is None:
                            r.first_token_s = now
                finished = [e for e in active if e[2] == len(e[0].prompt) and len(e[0].output) >= e[0].max_tokens]
                for e in finished:
                    e[0].done_s = now
                    self.model._drop_sequence(e[1])
                    held -= self._blocks(e[0])
                    active.remove(e)
        except BaseException:
            for e in active:
                try:
                    self.model._drop_sequence(e[1])
                except Exception:
                    pass
            raise
        return requests


def synthetic_requests(count: int, vocab: int, prompt=(32, 1024), output=(16, 256), seed: int = 0) -> list:
    """Seeded requests with prompt and output lengths uniform in the given
    inclusive ranges (the SmolLM2 serving workload's shape)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    plen = rng.integers(prompt[0], prompt[1] + 1, count)
    olen = rng.integers(output[0], output[1] + 1, count)
    return [ServeRequest(f"request-{i}", rng.integers(0, vocab, int(plen[i])).tolist(), int(olen[i]))
            for i in range(count)]
