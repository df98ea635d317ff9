"""Host-side checks that need no GPU: the library loads and exports every
declared symbol, the engine's KV accounting replays bit-exactly against the
reference's (kv.hpp), the GGUF writer/reader round-trips, and opening a model
without a CUDA device fails with an error instead of falling back."""

import ctypes as C
import re

import numpy as np
import pytest

from tests.conftest import ROOT
from tests.test_oracle_pins import _replay, ref_book, orc_book
from tvara_b200 import gguf


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"TVARA_API[^;(]*?\b(tvara_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol(capi):
    names = declared_symbols()
    assert len(names) >= 45
    missing = [n for n in names if not hasattr(capi, n)]
    assert not missing, missing


def test_reference_abi_is_exported_unchanged(capi):
    # core/include/tvara/c_api.h:13-24
    for n in ("tvara_model_open", "tvara_model_close", "tvara_model_vocab_size", "tvara_model_context_size",
              "tvara_last_error", "tvara_model_metadata", "tvara_sequence_create", "tvara_sequence_decode",
              "tvara_sequence_drop", "tvara_sequence_decode_batch", "tvara_sequence_truncate"):
        assert hasattr(capi, n)


def engine_book(L, blocks, tpb):
    b = L.tvara_kv_book_new(1, 1, 4, tpb, blocks)
    assert b

    def state(live):
        tables = {}
        for s in live:
            ids = (C.c_uint64 * 4096)()
            gens = (C.c_uint64 * 4096)()
            n = C.c_size_t()
            assert L.tvara_kv_book_table(b, s, ids, gens, 4096, C.byref(n)) == 0
            length = [x for x in (n.value,)]
            tables[s] = [(ids[i], gens[i]) for i in range(n.value)]
        avail = L.tvara_kv_book_available(b)
        return avail, [L.tvara_kv_book_references(b, i) for i in range(blocks)], tables

    lengths = {}

    def length(s):
        # replay bookkeeping via truncate-to-self: the table length is enough
        return lengths.get(s, 0)

    def wrap_append(s):
        r = L.tvara_kv_book_append(b, s)
        if r == 0:
            lengths[s] = lengths.get(s, 0) + 1
        return r

    def wrap_fork(s):
        i = L.tvara_kv_book_fork(b, s)
        if i:
            lengths[i] = lengths.get(s, 0)
        return i

    def wrap_truncate(s, n):
        r = L.tvara_kv_book_truncate(b, s, n)
        if r == 0:
            lengths[s] = n
        return r

    def wrap_import(s, n):
        i = L.tvara_kv_book_import(b, s, n)
        if i:
            lengths[i] = n
        return i

    def wrap_create():
        i = L.tvara_kv_book_create(b)
        lengths[i] = 0
        return i

    return dict(create=wrap_create, append=wrap_append, fork=wrap_fork, truncate=wrap_truncate,
                drop=lambda s: L.tvara_kv_book_drop(b, s), length=length, state=state,
                audit=lambda: L.tvara_kv_book_audit(b), **{"import": wrap_import})


def _strip_lengths(book):
    inner = book["state"]

    def state(live):
        avail, refs, tables = inner(live)
        return avail, refs, {s: [e for e in t if isinstance(e, tuple)] for s, t in tables.items()}

    book = dict(book)
    book["state"] = state
    return book


@pytest.mark.parametrize("blocks,tpb,seed", [(8, 2, 0), (16, 3, 1), (64, 16, 2), (5, 4, 3), (40, 7, 4)])
def test_engine_kv_accounting_bit_exact(capi, oracle_lib, blocks, tpb, seed):
    """Engine accounting == reference accounting (ids, generations, reference
    counts, free blocks) after every op; the reference is the compiled one when
    present, else the pinned C restatement."""
    from oracle import oracle as O
    ref = O.ref()
    other = ref_book(ref, blocks, tpb) if ref is not None else orc_book(oracle_lib, blocks, tpb)
    _replay([_strip_lengths(other), _strip_lengths(engine_book(capi, blocks, tpb))], seed, steps=300)


def test_engine_kv_book_known_answers(capi):
    # tests/core/test_kv.cpp:41-43: exhaustion leaves the branch unchanged
    L = capi
    b = L.tvara_kv_book_new(1, 1, 2, 2, 1)
    s = L.tvara_kv_book_create(b)
    assert L.tvara_kv_book_append(b, s) == 0
    br = L.tvara_kv_book_fork(b, s)
    assert L.tvara_kv_book_append(b, br) == -2  # copy-on-write needs a block: exhausted
    assert b"KV cache exhausted" in L.tvara_last_error()
    assert L.tvara_kv_book_references(b, 0) == 2
    assert L.tvara_kv_book_drop(b, br) == 0
    assert L.tvara_kv_book_append(b, s) == 0
    assert L.tvara_kv_book_drop(b, s) == 0
    assert L.tvara_kv_book_available(b) == 1
    assert L.tvara_kv_book_audit(b) == 0
    assert L.tvara_kv_book_drop(b, 99) == -1 and b"unknown KV sequence" in L.tvara_last_error()
    L.tvara_kv_book_free(b)


def test_gguf_writer_reader_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    for kind in (gguf.F32, gguf.F16, gguf.Q8_0, gguf.Q4_0, gguf.Q4_K):
        path = gguf.write_gguf(tmp_path / f"t{kind}.gguf", [("general.architecture", "str", "llama"),
                                                           ("x.u", "u32", 7), ("x.f", "f32", 0.5)],
                               [("w", kind, w.shape, gguf.encode(kind, w))])
        f = gguf.GGUFFile(path)
        assert f.metadata["x.u"] == 7 and f.metadata["x.f"] == 0.5
        assert f.kind("w") == kind and f.shape("w") == (64, 256)
        from oracle.oracle import dequantize
        back = dequantize(kind, f.raw("w"), w.size).reshape(w.shape)
        tol = {gguf.F32: 0, gguf.F16: 1e-4, gguf.Q8_0: 4e-4, gguf.Q4_0: 8e-3, gguf.Q4_K: 8e-3}[kind]
        assert np.abs(back - w).max() <= tol + 1e-9


def test_open_without_gpu_fails_loudly(capi, tiny_path):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present; covered by the GPU suite")
    except ImportError:
        pass
    h = capi.tvara_model_open(str(tiny_path).encode(), 16, 16)
    assert not h
    msg = capi.tvara_last_error().decode()
    assert "CUDA" in msg or "cuda" in msg


def test_open_rejects_bad_files_like_reference(capi, tmp_path):
    """Errors raised before any device work carry the reference's texts
    (gguf.hpp / gguf_model.hpp); this does not need a GPU."""
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 64)
    assert not capi.tvara_model_open(str(bad).encode(), 4, 4)
    # on a CPU box the CUDA device query may fail first; either is a loud error
    msg = capi.tvara_last_error().decode()
    assert msg
    assert not capi.tvara_model_open(b"", 4, 4)
    assert capi.tvara_last_error().decode() == "empty model path"
