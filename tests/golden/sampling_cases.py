"""Sampling cases of tests/golden/sampling.npz (made by make_golden.py from
the reference's NativeModel.iter_tokens) and the token constraint they use."""

import numpy as np


class EvenTokens:
    """A token constraint with the reference's interface (token_masks.py:
    228-246): only even token ids; accept records the tokens."""

    def __init__(self, vocab):
        self.vocab = vocab
        self.accepted = []

    def mask_logits(self, logits):
        values = np.asarray(logits, dtype=float)
        out = np.full(values.shape, -np.inf)
        out[0::2] = values[0::2]
        return out

    def accept(self, token):
        if token % 2:
            raise ValueError("token outside the constraint")
        self.accepted.append(token)


SAMPLING_CASES = {
    # name: iter_tokens keyword arguments (prompt: tiny_prompt()[:24], 32 new tokens)
    "greedy_penalties": dict(temperature=0, repetition=1.3, frequency=0.2, presence=0.3),
    "greedy_constraint": dict(temperature=0, repetition=0.7, presence=-0.1, constraint=True),
    "topk_penalties": dict(temperature=0.8, seed=7, top_k=8, min_p=0.05, top_p=0.9, repetition=1.1,
                           frequency=0.1),
    "topk_constraint": dict(temperature=1.2, seed=11, top_k=5, constraint=True),
}
