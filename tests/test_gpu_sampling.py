"""Device-side logit post-processing (k_sample.cu) against the restated
reference sampler (oracle/sampler.py, pinned to the reference's own
iter_tokens by tests/test_sampling_oracle.py).  Penalties, mask, checks,
argmax and top-k are float64 IEEE operations: everything is compared bit for
bit.  Generation through NativeModel.iter_tokens reproduces the reference's
golden tokens."""

import ctypes as C

import numpy as np
import pytest

from tests.conftest import GOLDEN
from tests.golden.sampling_cases import SAMPLING_CASES, EvenTokens
from tests.test_gpu_kernels import check, dev, ptr, sync, torch_dev

pytestmark = pytest.mark.gpu


def oracle_rows(logits, histories, params, allowed, k):
    from oracle import sampler as S
    out = []
    for r in range(len(logits)):
        rep, fre, pre = params[r]
        adj = S.adjust(logits[r], histories[r], rep, fre, pre)
        al = None if allowed is None else allowed[r]
        st = S.status(logits[r], adj, al)
        m = S.mask(adj, al)
        ids, vals = S.top_candidates(m, k)
        out.append((st, int(m.argmax()), ids, vals))
    return out


def make_case(rng, rows, vocab):
    logits = (rng.standard_normal((rows, vocab)) * 4).astype(np.float32)
    histories, params = [], []
    for r in range(rows):
        n = int(rng.choice([0, 1, 5, 300, 3000]))
        hot = rng.integers(0, vocab, 12)  # repeated tokens
        h = np.where(rng.random(n) < 0.5, rng.choice(hot, n), rng.integers(0, vocab, n))
        histories.append(h.astype(np.int32))
        params.append((float(rng.choice([1.0, 1.3, 0.7])), float(rng.choice([0.0, 0.2, -0.1])),
                       float(rng.choice([0.0, 0.5, -0.3]))))
    # special rows: ties for the maximum, signed zeros, a NaN, an infinity,
    # an adjusted value that overflows
    logits[0, [3, 7, 11]] = 50.0
    logits[1, :] = np.where(rng.random(vocab) < 0.5, -0.0, 0.0).astype(np.float32)
    logits[2, vocab // 2] = np.nan
    logits[3, 1] = np.inf
    logits[4, 5] = 3e38
    histories[4] = np.array([5, 5, 9], np.int32)
    params[4] = (1e-300, 0.0, 0.0)
    return logits, histories, params


@pytest.mark.parametrize("vocab", [512, 50001, 128256])
@pytest.mark.parametrize("k", [0, 1, 7, 64])
@pytest.mark.parametrize("masked", [False, True])
def test_sample_logits_kernel_bit_exact(capi, vocab, k, masked):
    torch = torch_dev()
    rng = np.random.default_rng(vocab + 10 * k + masked)
    rows = 12
    logits, histories, params = make_case(rng, rows, vocab)
    allowed = None
    if masked:
        allowed = rng.random((rows, vocab)) < 0.5
        allowed[6] = False
        allowed[6, vocab - 1] = True  # a single allowed token
        allowed[7] = False            # none allowed
    offs = np.zeros(rows + 1, np.uint64)
    np.cumsum([len(h) for h in histories], out=offs[1:])
    flat = np.concatenate(histories + [np.zeros(1, np.int32)])
    rep = np.array([p[0] for p in params])
    fre = np.array([p[1] for p in params])
    pre = np.array([p[2] for p in params])
    words = None
    if allowed is not None:
        packed = np.packbits(allowed, axis=1, bitorder="little")
        packed = np.pad(packed, ((0, 0), (0, (-packed.shape[1]) % 4)))
        words = dev(np.ascontiguousarray(packed).view(np.uint32))
    d_logits, d_hist = dev(logits), dev(flat)
    am = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = torch.empty(rows, dtype=torch.int32, device="cuda")
    tv = torch.empty(max(rows * k, 1), dtype=torch.float64, device="cuda")
    ti = torch.empty(max(rows * k, 1), dtype=torch.int32, device="cuda")
    n = capi.tvara_sample_workspace(rows, max(len(h) for h in histories))
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    f64 = C.POINTER(C.c_double)
    check(capi, capi.tvara_sample_logits(
        ptr(d_logits), rows, vocab, ptr(d_hist), offs.ctypes.data_as(C.POINTER(C.c_uint64)),
        rep.ctypes.data_as(f64), fre.ctypes.data_as(f64), pre.ctypes.data_as(f64),
        ptr(words) if words is not None else None, k, ptr(am), ptr(st), ptr(tv) if k else None,
        ptr(ti) if k else None, ptr(ws), n, None))
    sync()
    am, st = am.cpu().numpy(), st.cpu().numpy()
    tv = tv.cpu().numpy()[:rows * k].reshape(rows, k)
    ti = ti.cpu().numpy()[:rows * k].reshape(rows, k)
    want = oracle_rows(logits, histories, params, allowed, k)
    for r, (ws_, wa, wi, wv) in enumerate(want):
        assert st[r] == ws_, r
        if ws_ & 3:
            continue  # the reference raises before using the values
        assert am[r] == wa, r
        if k:
            assert ti[r].tolist() == wi.tolist(), r
            assert np.array_equal(tv[r].view(np.uint64), wv.astype(np.float64).view(np.uint64)), r
    assert want[2][0] == 1 and want[3][0] == 1 and want[4][0] == 2  # the special rows are what they claim


def test_sample_workspace_and_argument_errors(capi):
    assert capi.tvara_sample_workspace(4, 16385) == 0
    assert capi.tvara_sample_workspace(4, 100) > 4 * 128 * 8
    offs = np.array([0, 0], np.uint64)
    status = capi.tvara_sample_logits(None, 1, 10, None, offs.ctypes.data_as(C.POINTER(C.c_uint64)), None, None,
                                      None, None, 0, None, None, None, None, None, 0, None)
    assert status != 0 and b"invalid sampling arguments" in capi.tvara_last_error()


# ------------------------------------------------------------------ engine path
@pytest.fixture(scope="module")
def tiny(tiny_path):
    from tvara_b200.native import NativeModel
    with NativeModel(tiny_path, max_blocks=64, block_tokens=16) as m:
        yield m


@pytest.mark.parametrize("name", sorted(SAMPLING_CASES))
def test_iter_tokens_reproduce_reference_golden(tiny, name):
    g = np.load(GOLDEN / "sampling.npz")
    kw = dict(SAMPLING_CASES[name])
    constraint = EvenTokens(tiny.vocab_size) if kw.pop("constraint", False) else None
    toks = tiny.generate([int(t) for t in g["prompt"]], max_new_tokens=len(g[name]), token_constraint=constraint,
                         **kw)
    assert toks == g[name].tolist()


def test_greedy_fast_path_matches_sampler_path(tiny):
    """Plain greedy generation (temperature 0, default penalties, no
    constraint) runs one tvara_batch_step per token with the device's
    finite-checked argmax; the general path (tvara_batch_sample) gives the
    same tokens, and both stop at the same EOS."""
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, tiny.vocab_size, 37)]
    fast = tiny.generate(prompt, max_new_tokens=48)
    slow = list(tiny._iter_tokens_device(prompt, 48, 0.0, None, None, 1.0, 0, 0.0, 1.0, 0.0, 0.0, None))
    assert fast == slow and len(fast) == 48
    eos = fast[20]
    stop = fast.index(eos) + 1
    assert tiny.generate(prompt, max_new_tokens=48, eos_id=eos) == fast[:stop]
    assert tiny.generate(prompt, max_new_tokens=0) == []


def test_iter_tokens_argument_errors(tiny):
    """The reference's checks and texts (python/tvara/native.py:220-262)."""
    cases = [(dict(prompt=[]), "Invalid prompt token IDs"), (dict(prompt=[True]), "Invalid prompt token IDs"),
             (dict(prompt=[tiny.vocab_size]), "Invalid prompt token IDs"),
             (dict(max_new_tokens=10 ** 9), "Generation exceeds context limits"),
             (dict(max_new_tokens=1.0), "Generation exceeds context limits"),
             (dict(temperature="0"), "Sampling parameters must be real scalars"),
             (dict(top_p=True), "Sampling parameters must be real scalars"),
             (dict(temperature=-1), "Invalid sampling parameters"), (dict(top_p=0), "Invalid sampling parameters"),
             (dict(min_p=1.5), "Invalid sampling parameters"), (dict(top_k=-1), "Invalid sampling filters"),
             (dict(repetition=0), "Invalid sampling filters"), (dict(frequency=np.inf), "Invalid sampling filters"),
             (dict(eos_id=tiny.vocab_size), "Invalid EOS ID"), (dict(seed=True), "Invalid random seed"),
             (dict(seed=-1), "Invalid random seed"),
             (dict(temperature=0.5, top_k=0), "device sampling needs")]
    for kw, msg in cases:
        prompt = kw.pop("prompt", [1, 2])
        with pytest.raises(ValueError, match=msg):
            tiny.generate(prompt, **kw)


def test_batch_sample_histories_forks_and_masks(tiny):
    """Several sequences in one step with their own penalties and masks; the
    history of a fork includes its parent's tokens (copied tail ids), and
    reserved positions hold no token.  Compared with the oracle sampler over
    the same call's logits, bit for bit."""
    rng = np.random.default_rng(3)
    V = tiny.vocab_size
    prompts = [rng.integers(0, V, n).tolist() for n in (9, 17, 1)]
    seqs = [tiny._new_sequence() for _ in prompts]
    hist = [list(p) for p in prompts]
    k = 9
    out = tiny.batch_sample(seqs, prompts, repetition=[1.3, 0.8, 1.0], frequency=[0.1, 0.0, -0.2],
                            presence=[0.0, 0.4, 0.1], top_k=k, logits=True)
    fork = tiny.fork(seqs[0])
    hist.append(list(hist[0]))
    tiny.reserve(seqs[2], 3)  # positions without tokens
    seqs.append(fork)
    for step in range(4):
        toks = [[int(t)] for t in rng.integers(0, V, len(seqs))]
        for h, t in zip(hist, toks):
            h.extend(t)
        allowed = rng.random((len(seqs), V)) < 0.3
        params = [(float(rng.choice([1.0, 1.2])), float(rng.choice([0.0, 0.3])), float(rng.choice([0.0, -0.2])))
                  for _ in seqs]
        out = tiny.batch_sample(seqs, toks, [p[0] for p in params], [p[1] for p in params], [p[2] for p in params],
                                allowed, top_k=k, logits=True)
        want = oracle_rows(out["logits"], hist, params, allowed, k)
        for r, (ws_, wa, wi, wv) in enumerate(want):
            assert out["status"][r] == ws_
            assert out["argmax"][r] == wa
            assert out["top_ids"][r].tolist() == wi.tolist()
            assert np.array_equal(out["top_values"][r].view(np.uint64), wv.view(np.uint64))
    for s in seqs:
        tiny._drop_sequence(s)
    tiny.kv_audit()


def test_batch_sample_rejects_bad_arguments(tiny):
    s = tiny._new_sequence()
    with pytest.raises(RuntimeError, match="top-k"):
        tiny.batch_sample([s], [[1]], top_k=65)
    with pytest.raises(RuntimeError, match="Invalid sampling filters or penalties"):
        tiny.batch_sample([s], [[1]], repetition=0.0)
    assert tiny.sequence_length(s) == 0  # all-or-nothing: nothing appended
    tiny._drop_sequence(s)
