"""Owned ctypes handle over the B200 engine with the reference's
python/tvara/native.py:27-345 surface (same constructor, ``logits``,
``iter_tokens`` / ``generate`` sampled on the device, ``metadata`` and error
behaviour), plus the additive calls:
``decode_batch`` (multi-token append with rollback), ``batch_step`` (one
device step over a ragged batch of sequences), ``fork``, ``truncate``, KV
inspection and the radix prefix cache.
"""

from __future__ import annotations

import ctypes as C
import json
import threading
import weakref
from pathlib import Path

import numpy as np

from . import load_library
from ._bindings import OpenOptions, Sampling, F32P, F64P, U32P, U64P, I32P

KV_F32, KV_F16, KV_I8 = 0, 1, 2
STEP_ALL_LOGITS = 1
STEP_FINITE_ARGMAX = 2
ARGMAX_NONFINITE = 0xFFFFFFFF
SAMPLE_NONFINITE_LOGITS = 1
SAMPLE_NONFINITE_ADJUSTED = 2
SAMPLE_NONE_ALLOWED = 4
SAMPLE_MAX_K = 64
# Extra device candidates beyond top_k, so that tokens whose probabilities
# tie after rounding at the top_k boundary are still seen by the host.
SAMPLE_MARGIN = 16


def _ptr(a: np.ndarray, typ):
    return a.ctypes.data_as(typ)


def tp_shard(path, tp_rank: int, tp_size: int, library=None) -> dict:
    """tvara_tp_shard: the query heads, KV heads and FFN rows a tensor-parallel
    rank holds (reads the GGUF header only; no GPU needed)."""
    from ._bindings import TpShardInfo
    lib = load_library(library)
    info = TpShardInfo()
    info.struct_size = C.sizeof(TpShardInfo)
    if lib.tvara_tp_shard(str(Path(path).resolve()).encode("utf-8"), int(tp_rank), int(tp_size), C.byref(info)):
        raise RuntimeError(lib.tvara_last_error().decode("utf-8", "replace"))
    return {name: int(getattr(info, name)) for name, _ in TpShardInfo._fields_ if name != "struct_size"}


def _is_flag(v) -> bool:
    return isinstance(v, (bool, np.bool_))


def _is_int(v) -> bool:
    return isinstance(v, (int, np.integer)) and not _is_flag(v)


def _is_pyint(v) -> bool:
    return isinstance(v, int) and not _is_flag(v)


class _GenerationSettings:
    """Checked generation arguments.  Checks run in the reference's order and
    raise its texts (python/tvara/native.py:220-262), so callers see the same
    errors for the same bad input."""

    def __init__(self, vocab, context, prompt, max_new_tokens, temperature, seed, eos_id, top_p, top_k, min_p,
                 repetition, frequency, presence):
        self.prompt = list(prompt)
        if not self.prompt or not all(_is_int(t) and 0 <= t < vocab for t in self.prompt):
            raise ValueError("Invalid prompt token IDs")
        if not (_is_pyint(max_new_tokens) and 0 <= max_new_tokens <= context - len(self.prompt)):
            raise ValueError("Generation exceeds context limits")
        self.max_new_tokens = max_new_tokens
        reals = {}
        for name, v in (("temperature", temperature), ("top_p", top_p), ("min_p", min_p),
                        ("repetition", repetition), ("frequency", frequency), ("presence", presence)):
            if _is_flag(v) or not isinstance(v, (int, float, np.integer, np.floating)):
                raise ValueError("Sampling parameters must be real scalars")
            reals[name] = float(v)
        self.temperature, self.top_p, self.min_p = reals["temperature"], reals["top_p"], reals["min_p"]
        self.repetition, self.frequency, self.presence = reals["repetition"], reals["frequency"], reals["presence"]
        finite = np.isfinite
        if not (finite(self.temperature) and self.temperature >= 0 and finite(self.top_p) and 0 < self.top_p <= 1
                and finite(self.min_p) and 0 <= self.min_p <= 1):
            raise ValueError("Invalid sampling parameters")
        if not (_is_pyint(top_k) and top_k >= 0 and finite(self.repetition) and self.repetition > 0
                and finite(self.frequency) and finite(self.presence)):
            raise ValueError("Invalid sampling filters or penalties")
        self.top_k = top_k
        if eos_id is not None and not (_is_int(eos_id) and 0 <= eos_id < vocab):
            raise ValueError("Invalid EOS ID")
        self.eos_id = eos_id
        if _is_flag(seed):
            raise ValueError("Invalid random seed")
        try:
            self.rng = np.random.default_rng(seed)
        except (ValueError, TypeError, OverflowError) as error:
            raise ValueError("Invalid random seed") from error


class NativeModel:
    def __init__(self, path, library=None, max_blocks=256, block_tokens=16, *, kv_dtype=None, device=None,
                 max_step_tokens=None, tp_rank=0, tp_size=1, nccl_id: bytes | None = None, weight_planes=None):
        self._lock = threading.RLock()
        self._library = load_library(library)
        lib = self._library
        if (not isinstance(max_blocks, int) or not isinstance(block_tokens, int) or max_blocks <= 0
                or block_tokens <= 0):
            raise ValueError("Cache geometry must be positive integers")
        encoded = str(Path(path).resolve()).encode("utf-8")
        if kv_dtype is None and device is None and max_step_tokens is None and tp_size == 1 and weight_planes is None:
            self._handle = lib.tvara_model_open(encoded, max_blocks, block_tokens)
        else:
            opts = OpenOptions()
            opts.struct_size = C.sizeof(OpenOptions)
            opts.device = -1 if device is None else int(device)
            opts.kv_dtype = {None: KV_F32, "f32": KV_F32, "f16": KV_F16, "i8": KV_I8, KV_F32: KV_F32, KV_F16: KV_F16,
                             KV_I8: KV_I8}[kv_dtype]
            opts.max_step_tokens = int(max_step_tokens or 0)
            opts.tp_rank, opts.tp_size = int(tp_rank), int(tp_size)
            opts.weight_planes = {None: 0, "auto": 0, True: 1, "on": 1, False: 2, "off": 2, "hilo": 3,
                                  "q4kplane": 4}[weight_planes]
            self._nccl_id = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
            opts.nccl_id = C.cast(self._nccl_id, C.c_void_p) if self._nccl_id is not None else None
            self._handle = lib.tvara_model_open_ex(encoded, max_blocks, block_tokens, C.byref(opts))
        if not self._handle:
            self._raise_error()
        self._finalizer = weakref.finalize(self, lib.tvara_model_close, self._handle)
        self.vocab_size = int(lib.tvara_model_vocab_size(self._handle))
        self.context_size = int(lib.tvara_model_context_size(self._handle))
        self._tokenizer = None

    # ------------------------------------------------------------- lifecycle
    def _raise_error(self):
        message = self._library.tvara_last_error()
        raise RuntimeError(message.decode("utf-8", errors="replace") if message else "Native operation failed")

    def _check_open(self):
        if not self._handle:
            raise RuntimeError("Model is closed")

    def close(self):
        with self._lock:
            if self._handle:
                self._finalizer()
                self._handle = None

    def __enter__(self):
        self._check_open()
        return self

    def __exit__(self, *args):
        self.close()

    @property
    def metadata(self):
        with self._lock:
            self._check_open()
            raw = self._library.tvara_model_metadata(self._handle)
            if not raw:
                self._raise_error()
            return json.loads(raw.decode("utf-8"))

    # ------------------------------------------------------------- sequences
    def _new_sequence(self):
        with self._lock:
            self._check_open()
            seq = self._library.tvara_sequence_create(self._handle)
            if not seq:
                self._raise_error()
            return seq

    def _drop_sequence(self, sequence):
        with self._lock:
            if self._handle and self._library.tvara_sequence_drop(self._handle, sequence):
                self._raise_error()

    def logits(self, sequence, token):
        if isinstance(token, (bool, np.bool_)) or not isinstance(token, (int, np.integer)) \
                or not 0 <= token < self.vocab_size:
            raise ValueError("Invalid token ID")
        out = np.empty(self.vocab_size, dtype=np.float32)
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_decode(self._handle, sequence, int(token), _ptr(out, F32P), len(out)):
                self._raise_error()
        return out

    def decode_batch(self, sequence, tokens) -> np.ndarray:
        """tvara_sequence_decode_batch: every row's logits, rollback on failure."""
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty((len(toks), self.vocab_size), dtype=np.float32)
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_decode_batch(self._handle, sequence, _ptr(toks, U32P), len(toks),
                                                         _ptr(out, F32P), out.size):
                self._raise_error()
        return out

    def weight_bytes(self) -> dict:
        """Device bytes of the packed weights and of the FP16 weight planes."""
        packed, planes = C.c_size_t(), C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_model_weight_bytes(self._handle, C.byref(packed), C.byref(planes)):
                self._raise_error()
        return {"packed": packed.value, "planes": planes.value}

    def truncate(self, sequence, length):
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_truncate(self._handle, sequence, int(length)):
                self._raise_error()

    def fork(self, sequence):
        with self._lock:
            self._check_open()
            seq = self._library.tvara_sequence_fork(self._handle, sequence)
            if not seq:
                self._raise_error()
            return seq

    def sequence_length(self, sequence) -> int:
        n = C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_length(self._handle, sequence, C.byref(n)):
                self._raise_error()
        return n.value

    @staticmethod
    def _pack(sequences, token_lists):
        seqs = np.ascontiguousarray(sequences, dtype=np.uint64)
        if isinstance(token_lists, np.ndarray) and token_lists.ndim == 1:
            # decode: one token per sequence
            if len(token_lists) != len(seqs):
                raise ValueError("one token per sequence expected")
            toks = np.ascontiguousarray(token_lists, dtype=np.uint32)
            cu = np.arange(len(seqs) + 1, dtype=np.uint32)
        else:
            lens = np.array([len(t) for t in token_lists], dtype=np.uint32)
            cu = np.zeros(len(seqs) + 1, dtype=np.uint32)
            np.cumsum(lens, out=cu[1:])
            toks = np.ascontiguousarray(np.concatenate([np.asarray(t, dtype=np.uint32) for t in token_lists]))
        return seqs, cu, toks

    def batch_sample(self, sequences, token_lists, repetition=None, frequency=None, presence=None, allowed=None,
                     top_k=0, logits=False):
        """A step (one row per sequence) followed by the sampler's logit
        post-processing on the device (tvara_batch_sample): penalties from
        each sequence's tokens, the allowed-token mask ([n, vocab] bool or
        None), argmax and the top_k largest adjusted values.  Returns a dict
        of numpy arrays: argmax [n], status [n] (SAMPLE_* bits), top_values
        [n, top_k] float64, top_ids [n, top_k] and, with logits, the rows
        before post-processing [n, vocab] F32."""
        seqs, cu, toks = self._pack(sequences, token_lists)
        n = len(seqs)

        def per_row(v):
            if v is None:
                return None
            a = np.broadcast_to(np.asarray(v, dtype=np.float64), (n,))
            return np.ascontiguousarray(a)

        rep, fre, pre = per_row(repetition), per_row(frequency), per_row(presence)
        words = None
        if allowed is not None:
            mask = np.asarray(allowed, dtype=bool).reshape(n, self.vocab_size)
            words = np.packbits(mask, axis=1, bitorder="little")
            pad = (-words.shape[1]) % 4
            words = np.ascontiguousarray(np.pad(words, ((0, 0), (0, pad)))).view(np.uint32)
        args = Sampling()
        args.struct_size = C.sizeof(Sampling)
        args.repetition = _ptr(rep, F64P) if rep is not None else None
        args.frequency = _ptr(fre, F64P) if fre is not None else None
        args.presence = _ptr(pre, F64P) if pre is not None else None
        args.allowed = _ptr(words, U32P) if words is not None else None
        args.top_k = int(top_k)
        am = np.empty(n, dtype=np.uint32)
        st = np.empty(n, dtype=np.int32)
        tv = np.empty((n, top_k), dtype=np.float64)
        ti = np.empty((n, top_k), dtype=np.uint32)
        lg = np.empty((n, self.vocab_size), dtype=np.float32) if logits else None
        with self._lock:
            self._check_open()
            status = self._library.tvara_batch_sample(
                self._handle, n, _ptr(seqs, U64P), _ptr(cu, U32P), _ptr(toks, U32P), C.byref(args),
                _ptr(lg, F32P) if lg is not None else None, lg.size if lg is not None else 0,
                _ptr(am, U32P), _ptr(st, I32P), _ptr(tv, F64P) if top_k else None, _ptr(ti, U32P) if top_k else None)
            if status:
                self._raise_error()
        return {"argmax": am, "status": st, "top_values": tv, "top_ids": ti, "logits": lg}

    def batch_step(self, sequences, token_lists, all_logits=False, logits=True, argmax=False, finite_argmax=False):
        """One device step: sequence i appends token_lists[i] (or, given a 1-D
        array, the single token token_lists[i]).  Returns
        (logits [rows, vocab] or None, argmax [rows] or None) with one row per
        sequence (its last token) or per token when all_logits.  With
        finite_argmax, a row whose logits hold a NaN or an infinity has
        argmax ARGMAX_NONFINITE."""
        seqs, cu, toks = self._pack(sequences, token_lists)
        rows = int(cu[-1]) if all_logits else len(seqs)
        out = np.empty((rows, self.vocab_size), dtype=np.float32) if logits else None
        am = np.empty(rows, dtype=np.uint32) if argmax else None
        with self._lock:
            self._check_open()
            status = self._library.tvara_batch_step(
                self._handle, len(seqs), _ptr(seqs, U64P), _ptr(cu, U32P), _ptr(toks, U32P),
                (STEP_ALL_LOGITS if all_logits else 0) | (STEP_FINITE_ARGMAX if finite_argmax else 0),
                _ptr(out, F32P) if out is not None else None, out.size if out is not None else 0,
                _ptr(am, U32P) if am is not None else None, len(am) if am is not None else 0)
            if status:
                self._raise_error()
        return out, am

    # -------------------------------------------------------- device access
    @property
    def stream(self) -> int:
        """cudaStream_t (as an int) the handle's device work runs on."""
        with self._lock:
            self._check_open()
            s = self._library.tvara_model_stream(self._handle)
            if s is None:
                self._raise_error()
            return int(s)

    def kv_pool(self) -> dict:
        from ._bindings import C as _C

        class Info(_C.Structure):
            _fields_ = [("base", _C.c_void_p), ("max_blocks", _C.c_size_t), ("block_elements", _C.c_size_t),
                        ("kv_dtype", _C.c_uint32), ("layers", _C.c_uint32), ("kv_heads", _C.c_uint32),
                        ("head_dim", _C.c_uint32), ("block_tokens", _C.c_uint32)]

        info = Info()
        with self._lock:
            self._check_open()
            if self._library.tvara_kv_pool(self._handle, C.byref(info)):
                self._raise_error()
        out = {f: getattr(info, f) for f, _ in Info._fields_}
        if out["kv_dtype"] == KV_I8:
            scales = C.c_void_p()
            with self._lock:
                if self._library.tvara_kv_pool_scales(self._handle, C.byref(scales)):
                    self._raise_error()
            out["scales"] = scales.value  # one F32 per pool row (element offset / head_dim)
        return out

    def reserve(self, sequence, count):
        """Append `count` positions without computing their K/V."""
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_reserve(self._handle, sequence, int(count)):
                self._raise_error()

    # ------------------------------------------------------- KV inspection
    def kv_stats(self):
        a, m = C.c_size_t(), C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_kv_stats(self._handle, C.byref(a), C.byref(m)):
                self._raise_error()
        return a.value, m.value

    def kv_audit(self):
        with self._lock:
            self._check_open()
            if self._library.tvara_kv_audit(self._handle):
                self._raise_error()

    def sequence_blocks(self, sequence):
        n = C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_sequence_blocks(self._handle, sequence, None, None, 0, C.byref(n)):
                self._raise_error()
            ids = np.empty(n.value, np.uint64)
            gens = np.empty(n.value, np.uint64)
            if self._library.tvara_sequence_blocks(self._handle, sequence, _ptr(ids, U64P), _ptr(gens, U64P),
                                                   n.value, C.byref(n)):
                self._raise_error()
        return list(zip(ids.tolist(), gens.tolist()))

    def kv_references(self, block_id) -> int:
        r = C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_kv_references(self._handle, block_id, C.byref(r)):
                self._raise_error()
        return r.value

    # --------------------------------------------------------- prefix cache
    def prefix_insert(self, tokens, sequence) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        with self._lock:
            self._check_open()
            node = self._library.tvara_prefix_insert(self._handle, _ptr(t, I32P), len(t), sequence)
            if not node:
                self._raise_error()
        return node

    def prefix_reuse(self, tokens, partial=False):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = C.c_size_t()
        with self._lock:
            self._check_open()
            seq = self._library.tvara_prefix_reuse(self._handle, _ptr(t, I32P), len(t), int(bool(partial)),
                                                   C.byref(n))
            if not seq:
                self._raise_error()
        return seq, n.value

    def prefix_lookup(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        node, n = C.c_uint64(), C.c_size_t()
        with self._lock:
            self._check_open()
            if self._library.tvara_prefix_lookup(self._handle, _ptr(t, I32P), len(t), C.byref(node), C.byref(n)):
                self._raise_error()
        return node.value, n.value

    def _prefix_call(self, name, node):
        with self._lock:
            self._check_open()
            if getattr(self._library, name)(self._handle, node):
                self._raise_error()

    def prefix_pin(self, node):
        self._prefix_call("tvara_prefix_pin", node)

    def prefix_unpin(self, node):
        self._prefix_call("tvara_prefix_unpin", node)

    def prefix_touch(self, node):
        self._prefix_call("tvara_prefix_touch", node)

    def prefix_evict_one(self) -> bool:
        with self._lock:
            self._check_open()
            r = self._library.tvara_prefix_evict_one(self._handle)
            if r < 0:
                self._raise_error()
        return bool(r)

    def prefix_size(self) -> int:
        with self._lock:
            self._check_open()
            return int(self._library.tvara_prefix_size(self._handle))

    # ------------------------------------------------------------ generation
    def iter_tokens(self, prompt, max_new_tokens=16, temperature=0, seed=0, eos_id=None, top_p=1, top_k=0,
                    min_p=0, repetition=1, frequency=0, presence=0, token_constraint=None):
        """Generation with the reference's arguments, errors and tokens
        (python/tvara/native.py:220-340), sampled on the device: the penalties,
        the token constraint's mask, the finiteness checks and either the
        argmax (temperature 0: the reference's token bit for bit) or the
        top_k + 16 largest adjusted logits are computed by tvara_batch_sample,
        and only those cross to the host, where numpy draws the token.  On the
        candidate path the probabilities are normalised over the candidates
        rather than the whole vocabulary, which changes them by rounding
        only: the drawn token can differ only if the uniform draw falls within
        that rounding of a boundary of the cumulative distribution.

        Settings the device does not cover -- temperature > 0 with top_k 0 or
        above 48 -- raise ValueError; the reference's own NativeModel, loaded
        on this library through TVARA_LIBRARY, samples those on the host."""
        s = _GenerationSettings(self.vocab_size, self.context_size, prompt, max_new_tokens, temperature, seed,
                                eos_id, top_p, top_k, min_p, repetition, frequency, presence)
        if not (s.temperature == 0 or 1 <= s.top_k <= SAMPLE_MAX_K - SAMPLE_MARGIN):
            raise ValueError("device sampling needs temperature 0 or 1 <= top_k <= 48; use the reference "
                             "NativeModel on this library for other settings")
        if s.temperature == 0 and token_constraint is None and (s.repetition, s.frequency, s.presence) == (1, 0, 0):
            # plain greedy decoding: the adjusted logits are the logits, so the
            # step's own finite-checked argmax is the token
            yield from self._iter_greedy_device(s.prompt, s.max_new_tokens, s.eos_id)
            return
        yield from self._iter_tokens_device(s.prompt, s.max_new_tokens, s.temperature, s.rng, s.eos_id, s.top_p,
                                            s.top_k, s.min_p, s.repetition, s.frequency, s.presence,
                                            token_constraint)

    def _iter_greedy_device(self, prompt, max_new_tokens, eos_id):
        """Greedy tokens with default penalties and no constraint: one
        tvara_batch_step per token with the device argmax and its finiteness
        check (STEP_FINITE_ARGMAX), into arrays allocated once, so only the
        token crosses to the host.  Same tokens and errors as the sampler path
        (python/tvara/native.py:301-336 at temperature 0)."""
        sequence = self._new_sequence()
        try:
            seqs = np.array([sequence], dtype=np.uint64)
            feed = np.ascontiguousarray(prompt, dtype=np.uint32)
            cu = np.array([0, len(feed)], dtype=np.uint32)
            nxt = np.zeros(1, dtype=np.uint32)
            cu1 = np.array([0, 1], dtype=np.uint32)
            am = np.empty(1, dtype=np.uint32)
            p_seq, p_am = _ptr(seqs, U64P), _ptr(am, U32P)
            p_cu, p_tok = _ptr(cu, U32P), _ptr(feed, U32P)
            for index in range(max_new_tokens):
                with self._lock:
                    self._check_open()
                    if self._library.tvara_batch_step(self._handle, 1, p_seq, p_cu, p_tok, STEP_FINITE_ARGMAX, None,
                                                      0, p_am, 1):
                        self._raise_error()
                token = int(am[0])
                if token == ARGMAX_NONFINITE:
                    raise ValueError("Nonfinite model logits")
                yield token
                if token == eos_id or index + 1 == max_new_tokens:
                    break
                nxt[0] = token
                p_cu, p_tok = _ptr(cu1, U32P), _ptr(nxt, U32P)
        finally:
            self._drop_sequence(sequence)

    def _iter_tokens_device(self, prompt, max_new_tokens, temperature, rng, eos_id, top_p, top_k, min_p, repetition,
                            frequency, presence, token_constraint):
        k = 0 if temperature == 0 else top_k + SAMPLE_MARGIN
        sequence = self._new_sequence()
        try:
            feed = prompt
            for index in range(max_new_tokens):
                allowed, mask_error = None, None
                if token_constraint is not None:
                    # the constraint's own mask (-inf outside its tokens); its error is
                    # raised after the logit checks, in the reference's order
                    try:
                        allowed = np.isfinite(token_constraint.mask_logits(np.zeros(self.vocab_size)))[None, :]
                    except ValueError as error:
                        mask_error = error
                out = self.batch_sample([sequence], [feed], repetition, frequency, presence, allowed, k)
                status = int(out["status"][0])
                if status & SAMPLE_NONFINITE_LOGITS:
                    raise ValueError("Nonfinite model logits")
                if status & SAMPLE_NONFINITE_ADJUSTED:
                    raise ValueError("Nonfinite adjusted sampling logits")
                if mask_error is not None:
                    raise mask_error
                if status & SAMPLE_NONE_ALLOWED:
                    raise ValueError("No grammar-valid tokens remain")
                if temperature == 0:
                    token = int(out["argmax"][0])
                else:
                    # the reference's filters on the candidates, held in token order
                    ids = out["top_ids"][0].astype(np.int64)
                    vals = out["top_values"][0]
                    order_ids = np.argsort(ids, kind="stable")
                    ids, vals = ids[order_ids], vals[order_ids]
                    p = np.exp((vals - float(vals.max())) / temperature)
                    p /= p.sum()
                    order = np.argsort(-p, kind="stable")
                    p[order[top_k:]] = 0
                    p[p < p.max() * min_p] = 0
                    p /= p.sum()
                    cumulative = np.cumsum(p[order])
                    p[order[np.r_[False, cumulative[:-1] >= top_p]]] = 0
                    p /= p.sum()
                    full = np.zeros(self.vocab_size)
                    full[ids] = p
                    token = int(rng.choice(self.vocab_size, p=full))
                if token_constraint is not None:
                    token_constraint.accept(token)
                yield token
                if token == eos_id:
                    break
                feed = [token]
                if index + 1 == max_new_tokens:
                    break
        finally:
            self._drop_sequence(sequence)

    def generate(self, prompt, **options):
        return list(self.iter_tokens(prompt, **options))
