"""The sampler restatement (oracle/sampler.py) pinned against the reference's
own NativeModel.iter_tokens: the CPU oracle model with the restated penalties,
mask, filters and numpy draw reproduces tests/golden/sampling.npz."""

import numpy as np
import pytest

from tests.conftest import GOLDEN
from tests.golden.sampling_cases import SAMPLING_CASES, EvenTokens


def oracle_generate(model, prompt, count, temperature=0, seed=0, top_p=1, top_k=0, min_p=0, repetition=1,
                    frequency=0, presence=0, constraint=None):
    from oracle import sampler as S
    rng = np.random.default_rng(seed)
    state = model.new_state()
    history = list(prompt)
    for t in prompt:
        logits = model.decode(state, t)
    out = []
    for i in range(count):
        adjusted = S.adjust(logits, history, repetition, frequency, presence)
        if constraint is not None:
            adjusted = constraint.mask_logits(adjusted)
        if temperature == 0:
            token = int(adjusted.argmax())
        else:
            p = S.filter_probabilities(adjusted, temperature, top_k, min_p, top_p)
            token = int(rng.choice(len(adjusted), p=p))
        if constraint is not None:
            constraint.accept(token)
        history.append(token)
        out.append(token)
        if i + 1 < count:
            logits = model.decode(state, token)
    return out


@pytest.fixture(scope="module")
def oracle_tiny(tiny_path):
    from oracle.model import OracleModel
    return OracleModel(tiny_path, max_positions=128)


@pytest.mark.parametrize("name", sorted(SAMPLING_CASES))
def test_restated_sampler_reproduces_reference_tokens(oracle_tiny, name):
    g = np.load(GOLDEN / "sampling.npz")
    kw = dict(SAMPLING_CASES[name])
    constraint = EvenTokens(oracle_tiny.vocab) if kw.pop("constraint", False) else None
    got = oracle_generate(oracle_tiny, [int(t) for t in g["prompt"]], len(g[name]), constraint=constraint, **kw)
    assert got == g[name].tolist()


def test_top_candidates_order_and_masking():
    from oracle import sampler as S
    v = np.array([1.0, 3.0, 3.0, -np.inf, 2.0, 3.0, -0.0, 0.0])
    ids, vals = S.top_candidates(v, 7)
    # ties (including -0.0 and +0.0) by index
    assert ids.tolist() == [1, 2, 5, 4, 0, 6, 7] and vals.tolist() == [3.0, 3.0, 3.0, 2.0, 1.0, 0.0, 0.0]
    m = S.mask(v, np.array([True, False] * 4))
    assert np.isneginf(m[1::2]).all() and (m[0::2] == v[0::2]).all()
    assert S.status(np.array([1.0, np.nan]), v, None) == 1
    assert S.status(np.ones(2), np.array([1.0, np.inf]), np.array([False, False])) == 6


def test_generation_checks_match_reference():
    """The argument checks of NativeModel.iter_tokens raise what the
    reference's raise (python/tvara/native.py:220-262), for the same inputs
    in the same order; the reference's generator runs on a stand-in whose
    first model call stops it once its checks have passed."""
    from oracle import reference_module
    from tvara_b200.native import _GenerationSettings
    ref = reference_module("native")
    if ref is None:
        pytest.skip("reference Python package not staged (oracle/_ref/python)")

    class Passed(Exception):
        pass

    class Stub:
        vocab_size, context_size = 50, 40

        def _new_sequence(self):
            raise Passed()

    def outcome(fn):
        try:
            fn()
        except Passed:
            return "ok"
        except ValueError as e:
            return str(e)
        return "ok"

    values = [0, 1, -1, 2.5, True, np.bool_(False), np.int64(3), np.float32(0.5), "1", None, np.inf, np.nan, 10 ** 30,
              0.95, 49, 50]
    rng = np.random.default_rng(0)
    names = ["max_new_tokens", "temperature", "seed", "eos_id", "top_p", "top_k", "min_p", "repetition", "frequency",
             "presence"]
    for _ in range(3000):
        kw = {n: values[int(rng.integers(len(values)))] for n in names if rng.random() < 0.3}
        prompt = [[1, 2], [], [True], [49], [50], [np.int32(3)], [1.0]][int(rng.integers(7))]
        want = outcome(lambda: next(ref.NativeModel.iter_tokens(Stub(), prompt, **kw)))
        full = dict(max_new_tokens=16, temperature=0, seed=0, eos_id=None, top_p=1, top_k=0, min_p=0, repetition=1,
                    frequency=0, presence=0)
        full.update(kw)
        got = outcome(lambda: _GenerationSettings(Stub.vocab_size, Stub.context_size, prompt, **full))
        assert got == want, (prompt, kw, got, want)
