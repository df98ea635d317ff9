"""Model-level parity on the GPU through the engine's C ABI, against the
reference engine's own outputs (tests/golden/, produced by make_golden.py)
and the pinned numpy oracle.

Logit tolerance: max-abs 2e-3 and relative 1e-3 of the
reference's F32 CPU path; greedy token sequences identical."""

import numpy as np
import pytest

from tvara_b200 import gguf
from tvara_b200.native import NativeModel
from tests.conftest import GOLDEN, make_model

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def close(got, ref):
    got, ref = np.asarray(got), np.asarray(ref)
    return np.all(np.abs(got - ref) <= ATOL) and np.all(np.abs(got - ref) <= RTOL * np.abs(ref) + ATOL)


@pytest.fixture(scope="module")
def tiny(tiny_path):
    with NativeModel(tiny_path, max_blocks=64, block_tokens=16) as m:
        yield m


@pytest.fixture(scope="module")
def oracle_tiny(tiny_path):
    from oracle.model import OracleModel
    return OracleModel(tiny_path, max_positions=512)


def test_open_metadata_and_sizes(tiny, tiny_path):
    assert tiny.vocab_size == 512 and tiny.context_size == 2048
    md = tiny.metadata
    assert md["general.architecture"] == "llama" and md["llama.block_count"] == 4
    from oracle import oracle as O
    if O.ref_capi() is not None:
        from oracle.model import RefEngine
        ref = RefEngine(tiny_path)
        assert tiny._library.tvara_model_metadata(tiny._handle) == ref.L.tvara_model_metadata(ref.h)


def test_tiny_logits_match_reference_golden(tiny):
    """BASELINE tiny config: 64-token prompt + 64 greedy tokens, every
    position's logits within tolerance of the reference engine's."""
    g = np.load(GOLDEN / "tiny_q8.npz")
    toks = np.concatenate([g["prompt"], g["greedy"]]).tolist()
    s = tiny._new_sequence()
    got = np.stack([tiny.logits(s, t) for t in toks])
    tiny._drop_sequence(s)
    assert close(got, g["logits"]), np.abs(got - g["logits"]).max()


def test_tiny_greedy_matches_reference(tiny):
    g = np.load(GOLDEN / "tiny_q8.npz")
    assert tiny.generate(g["prompt"].tolist(), max_new_tokens=64) == g["greedy"].tolist()


def test_mixed_types_and_interleaved_rope_match_reference_golden(model_dir):
    from tests.golden.make_golden import MIXED
    g = np.load(GOLDEN / "tiny_mixed.npz")
    path = make_model(model_dir, "mixed", gguf.model_config("tiny", **MIXED), seed=3)
    with NativeModel(path, max_blocks=16, block_tokens=16) as m:
        s = m._new_sequence()
        got = np.stack([m.logits(s, int(t)) for t in g["tokens"]])
    assert close(got, g["logits"]), np.abs(got - g["logits"]).max()


def test_decode_batch_equals_token_by_token(tiny, oracle_tiny):
    rng = np.random.default_rng(4)
    toks = rng.integers(0, 512, 40).tolist()
    a = tiny._new_sequence()
    rows = tiny.decode_batch(a, toks)
    ref = oracle_tiny.forward(toks)
    assert close(rows, ref)
    b = tiny._new_sequence()
    single = np.stack([tiny.logits(b, t) for t in toks])
    assert np.abs(rows - single).max() < 1e-4
    assert tiny.sequence_length(a) == 40
    tiny._drop_sequence(a)
    tiny._drop_sequence(b)


def test_decode_batch_rollback_and_errors(tiny):
    s = tiny._new_sequence()
    tiny.decode_batch(s, [1, 2, 3])
    with pytest.raises(RuntimeError, match="invalid batch token"):
        tiny.decode_batch(s, [4, 512])
    assert tiny.sequence_length(s) == 3
    with pytest.raises(RuntimeError, match="batch exceeds context"):
        tiny.decode_batch(s, [1] * (tiny.context_size - 2))
    assert tiny.sequence_length(s) == 3
    with pytest.raises(ValueError):
        tiny.logits(s, 512)
    with pytest.raises(RuntimeError, match="unknown KV sequence"):
        tiny.logits(987654, 1)
    tiny.truncate(s, 1)
    assert tiny.sequence_length(s) == 1
    with pytest.raises(RuntimeError, match="cannot extend KV by truncating"):
        tiny.truncate(s, 5)
    tiny._drop_sequence(s)
    tiny.kv_audit()


def test_exhaustion_leaves_state_unchanged(tiny_path):
    """tests/core/test_kv.cpp:41-43 and c_api.cpp:69-70: a failing batch
    rolls back; the pool and the other sequence are untouched."""
    with NativeModel(tiny_path, max_blocks=3, block_tokens=4) as m:
        a = m._new_sequence()
        m.decode_batch(a, [1, 2, 3, 4, 5, 6, 7, 8])
        c = m._new_sequence()
        before = m.sequence_blocks(a), m.kv_stats()
        with pytest.raises(RuntimeError, match="KV cache exhausted"):
            m.decode_batch(c, [8, 9, 10, 11, 12])
        assert m.sequence_length(c) == 0 and m.sequence_blocks(c) == []
        assert (m.sequence_blocks(a), m.kv_stats()) == before
        with pytest.raises(RuntimeError, match="invalid paged KV append dimensions"):
            for t in range(5):  # 12 = max_blocks * block_tokens positions per sequence
                m.logits(a, t)
        assert m.sequence_length(a) == 12
        m._drop_sequence(a)
        m.decode_batch(c, [8, 9, 10])
        assert m.sequence_length(c) == 3
        m.kv_audit()


def test_ragged_batch_step_matches_oracle(tiny, oracle_tiny):
    """One step mixing prefill chunks and single decode tokens over several
    sequences equals each sequence run alone through the oracle."""
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 512, n).tolist() for n in (5, 17, 1, 33, 16)]
    seqs = [tiny._new_sequence() for _ in prompts]
    logits, am = tiny.batch_step(seqs, prompts, argmax=True)
    states = [oracle_tiny.new_state() for _ in prompts]
    for i, p in enumerate(prompts):
        last = None
        for t in p:
            last = oracle_tiny.decode(states[i], t)
        assert close(logits[i], last)
        assert am[i] == int(np.argmax(logits[i]))
    for step in range(6):
        nxt = [[int(a)] for a in am]
        if step % 2:
            nxt[1] = nxt[1] + rng.integers(0, 512, 9).tolist()  # a chunk mid-generation
        logits, am = tiny.batch_step(seqs, nxt, argmax=True)
        for i, toks in enumerate(nxt):
            for t in toks:
                last = oracle_tiny.decode(states[i], t)
            assert close(logits[i], last)
    all_rows, _ = tiny.batch_step(seqs[:2], [[3, 4], [5]], all_logits=True)
    assert all_rows.shape == (3, 512)
    for s in seqs:
        tiny._drop_sequence(s)
    tiny.kv_audit()


@pytest.mark.parametrize("types", [dict(default=gguf.Q4_K, ffn_down=gguf.Q4_K, output=gguf.Q8_0),
                                   dict(default=gguf.Q4_0, ffn_down=gguf.Q8_0, output=gguf.Q4_0)],
                         ids=["q4k", "q40_q80"])
def test_wide_decode_matches_oracle(model_dir, types):
    """Single-token decode steps of a model wide enough (hidden 1024, ffn
    2816) for the streamed GEMV: every projection -- QKV, O with the residual
    add, gate/up with SwiGLU, down, the LM head -- runs at one token."""
    from oracle.model import OracleModel
    cfg = gguf.model_config("tiny", hidden=1024, heads=8, kv_heads=2, ffn=2816, layers=2, tied=False,
                            types=dict(types, embd=gguf.Q8_0))
    path = make_model(model_dir, "wide_" + "_".join(str(v) for v in types.values()), cfg, seed=5)
    ref = OracleModel(path, max_positions=64)
    state = ref.new_state()
    rng = np.random.default_rng(4)
    with NativeModel(path, max_blocks=8, block_tokens=16) as m:
        seq = m._new_sequence()
        tok = int(rng.integers(0, 512))
        for _ in range(5):
            logits, am = m.batch_step([seq], [[tok]], argmax=True)
            want = ref.decode(state, tok)
            assert close(logits[0], want)
            tok = int(am[0])


def test_fork_copy_on_write(tiny, oracle_tiny):
    """kv.hpp fork + copy-on-write of a shared partial tail block: both
    branches keep their own continuation."""
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, 512, 21).tolist()
    a = tiny._new_sequence()
    tiny.decode_batch(a, prompt)
    b = tiny.fork(a)
    assert tiny.sequence_blocks(a) == tiny.sequence_blocks(b)
    shared = tiny.sequence_blocks(a)[-1][0]
    assert tiny.kv_references(shared) == 2
    la, _ = tiny.batch_step([a, b], [[7], [9]])
    assert tiny.sequence_blocks(a)[-1][0] != tiny.sequence_blocks(b)[-1][0]
    sa, sb = oracle_tiny.new_state(), None
    for t in prompt:
        oracle_tiny.decode(sa, t)
    sb = oracle_tiny.fork(sa)
    assert close(la[0], oracle_tiny.decode(sa, 7)) and close(la[1], oracle_tiny.decode(sb, 9))
    for s in (a, b):
        tiny._drop_sequence(s)
    tiny.kv_audit()


def test_radix_prefix_reuse_bit_identical(tiny):
    """tests/core/test_radix.cpp:22: logits after reusing a cached prefix are
    identical to a cold forward over the same tokens."""
    stem = [11, 22, 33, 44, 55, 66, 77, 88, 99, 10, 20, 30, 40, 50, 60, 70, 80, 90]
    src = tiny._new_sequence()
    for t in stem:
        tiny.logits(src, t)
    node = tiny.prefix_insert(stem, src)
    assert node and tiny.prefix_size() >= 1
    for tail in (4, 5, 6):
        seq, reused = tiny.prefix_reuse(stem + [tail], partial=True)
        assert reused == len(stem)
        cached = tiny.logits(seq, tail)
        cold_seq = tiny._new_sequence()
        for t in stem:
            tiny.logits(cold_seq, t)
        cold = tiny.logits(cold_seq, tail)
        assert np.array_equal(cached, cold)
        tiny._drop_sequence(seq)
        tiny._drop_sequence(cold_seq)
    full, reused = tiny.prefix_reuse(stem + [1], partial=False)
    assert reused == 16
    tiny._drop_sequence(full)
    tiny._drop_sequence(src)
    tiny.kv_audit()
    tiny.prefix_touch(node)
    assert tiny.prefix_evict_one()
    tiny.kv_audit()


def test_f16_kv_within_tolerance(tiny_path, oracle_tiny):
    g = np.load(GOLDEN / "tiny_q8.npz")
    toks = np.concatenate([g["prompt"], g["greedy"]]).tolist()
    with NativeModel(tiny_path, max_blocks=64, block_tokens=16, kv_dtype="f16") as m:
        s = m._new_sequence()
        got = m.decode_batch(s, toks)
    assert close(got, g["logits"]), np.abs(got - g["logits"]).max()


def test_small_step_budget_splits_long_prefill(tiny_path):
    """A prefill longer than max_step_tokens runs as several device steps with
    identical results."""
    g = np.load(GOLDEN / "tiny_q8.npz")
    toks = np.concatenate([g["prompt"], g["greedy"]]).tolist()
    with NativeModel(tiny_path, max_blocks=64, block_tokens=16, max_step_tokens=7) as m:
        s = m._new_sequence()
        got = m.decode_batch(s, toks)
    assert close(got, g["logits"])


@pytest.mark.parametrize("name", ["tiny", "mixed"])
def test_weight_planes_match_packed_path(tiny_path, model_dir, name):
    """Tensor-core batches read exact FP16 hi/lo planes when they are built and
    dequantise the packed rows otherwise: both stay within tolerance of the
    reference, and of each other to F32 rounding."""
    if name == "tiny":
        path, golden = tiny_path, np.load(GOLDEN / "tiny_q8.npz")
        toks = np.concatenate([golden["prompt"], golden["greedy"]]).tolist()
        want = golden["logits"]
    else:
        from tests.golden.make_golden import MIXED
        golden = np.load(GOLDEN / "tiny_mixed.npz")
        path = make_model(model_dir, "mixed", gguf.model_config("tiny", **MIXED), seed=3)
        toks, want = [int(t) for t in golden["tokens"]], golden["logits"]
    got = {}
    for planes in ("on", "off"):
        with NativeModel(path, max_blocks=64, block_tokens=16, weight_planes=planes) as m:
            sizes = m.weight_bytes()
            assert (sizes["planes"] > 0) == (planes == "on") and sizes["packed"] > 0
            s = m._new_sequence()
            got[planes] = m.decode_batch(s, toks)
        assert close(got[planes], want), (planes, np.abs(got[planes] - want).max())
    assert np.abs(got["on"] - got["off"]).max() <= 1e-4


@pytest.mark.parametrize("split_k", [False, True])
def test_wide_q4k_prefill_matches_oracle(model_dir, split_k):
    """Multi-token steps of a Q4_K model wide enough (K >= 1024, a multiple of
    256) for the two-MMA tensor-core form (FP16 plane of sc*q, block scales,
    min term): every position's logits within tolerance of the oracle, for the
    planes and for the packed path, and the two within 1e-4.  A short step
    budget splits the prompt across device steps; a single 48-token step uses
    split K on the narrow projections."""
    from oracle.model import OracleModel
    cfg = gguf.model_config("tiny", hidden=1024, heads=8, kv_heads=2, ffn=2816, layers=2, tied=False,
                            types=dict(default=gguf.Q4_K, ffn_down=gguf.Q4_K, output=gguf.Q8_0, embd=gguf.Q8_0))
    path = make_model(model_dir, "wide_q4k_prefill", cfg, seed=6)
    toks = np.random.default_rng(9).integers(0, 512, 48).tolist()
    want = OracleModel(path, max_positions=64).forward(toks)
    got = {}
    for planes in ("on", "off"):
        with NativeModel(path, max_blocks=8, block_tokens=16, weight_planes=planes,
                         max_step_tokens=None if split_k else 20) as m:
            assert (m.weight_bytes()["planes"] > 0) == (planes == "on")
            s = m._new_sequence()
            got[planes] = m.decode_batch(s, toks)
        assert close(got[planes], want), (planes, np.abs(got[planes] - want).max())
    assert np.abs(got["on"] - got["off"]).max() <= 1e-4


def test_batch_step_decode_array_equals_lists(tiny_path):
    """The 1-D decode form of batch_step (one token per sequence) is the same
    call as the list form."""
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 512, n).tolist() for n in (5, 9, 2)]
    outs = []
    for form in ("lists", "array"):
        with NativeModel(tiny_path, max_blocks=32, block_tokens=16) as m:
            seqs = [m._new_sequence() for _ in prompts]
            m.batch_step(seqs, prompts, logits=False)
            toks = np.array([7, 8, 9], dtype=np.uint32)
            arg = toks if form == "array" else [[int(t)] for t in toks]
            logits, am = m.batch_step(np.array(seqs, dtype=np.uint64), arg, argmax=True)
            outs.append((logits, am))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
