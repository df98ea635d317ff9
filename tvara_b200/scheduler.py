"""Scheduler backend that runs each scheduler iteration as one device step.

The reference's continuous-batching ``Scheduler`` (python/tvara/scheduler.py)
drives its model through a duck-typed backend with four calls: ``create``,
``prefill``, ``decode_batch`` and ``drop`` (scheduler.py:89-90, 107, 113, 127).
Its own ``NativeSchedulerBackend`` (scheduler.py:186-214) calls
``NativeModel.logits`` once per token per sequence.  ``BatchedSchedulerBackend``
is a drop-in for it: the reference's scheduler is used unchanged, and every
iteration becomes ONE ``tvara_batch_step`` -- the prefill chunks queued since
the last step and the token each decoding sequence emitted last time run
together on the device, and only the argmax of each sequence's last row comes
back (the finiteness check runs on the device too).

    from tvara.scheduler import Scheduler           # the reference's
    from tvara_b200.native import NativeModel
    from tvara_b200.scheduler import BatchedSchedulerBackend
    s = Scheduler(BatchedSchedulerBackend(NativeModel(path)), prefill_chunk=512)

Tokens returned are the ones the serial backend returns: the argmax of the
logits after the sequence's last fed token.
"""

from __future__ import annotations


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
