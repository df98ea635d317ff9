"""Test infrastructure only: a CPU restatement of the reference's sampler
(python/tvara/native.py:301-336, token_masks.py:228-241), the checker for the
device-side logit post-processing (k_sample.cu).  Nothing in the product
imports this module.  Pinned against the reference's own iter_tokens through
tests/golden/sampling.npz (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np


def adjust(logits, history, repetition=1.0, frequency=0.0, presence=0.0):
    """Penalised float64 logits: native.py:302 (float64 copy), :307-311
    (repetition on seen tokens, then count * frequency + seen * presence)."""
    values = np.asarray(logits).astype(np.float64, copy=True)
    counts = np.bincount(np.asarray(history, dtype=np.int64), minlength=len(values))
    seen = counts > 0
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        values[seen] = np.where(values[seen] >= 0, values[seen] / repetition, values[seen] * repetition)
        values -= counts * frequency + seen * presence
    return values


def mask(values, allowed):
    """token_masks.py:239-241: -inf outside the allowed tokens."""
    if allowed is None:
        return values
    out = np.full(values.shape, -np.inf)
    out[allowed] = values[allowed]
    return out


def status(logits, adjusted, allowed):
    """The reference's checks as device status bits: native.py:304-305
    (model logits), :312-313 (adjusted), token_masks.py:237-238 (mask)."""
    bits = 0
    if not np.isfinite(logits).all():
        bits |= 1
    elif not np.isfinite(adjusted).all():
        bits |= 2
    if allowed is not None and not np.asarray(allowed).any():
        bits |= 4
    return bits


def top_candidates(values, k):
    """The k largest values, value descending and index ascending on ties
    (the stable order of native.py:322 for distinct probabilities)."""
    order = np.lexsort((np.arange(len(values)), -values))
    return order[:k], values[order[:k]]


def filter_probabilities(values, temperature, top_k, min_p, top_p):
    """native.py:319-330: the probabilities rng.choice draws from."""
    p = np.exp((values.astype(float) - float(values.max())) / temperature)
    p /= p.sum()
    order = np.argsort(-p, kind="stable")
    if top_k:
        p[order[top_k:]] = 0
    p[p < p.max() * min_p] = 0
    p /= p.sum()
    cumulative = np.cumsum(p[order])
    p[order[np.r_[False, cumulative[:-1] >= top_p]]] = 0
    p /= p.sum()
    return p
