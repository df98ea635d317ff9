"""numpy restatement of the reference executor -- TEST INFRASTRUCTURE ONLY.

Follows core/include/tvara/paged_model.hpp:12-28 (decode) and the math in
model.hpp:49-126 / attention.hpp:6-83:

* embedding_lookup (model.hpp:49-55): the token's row, dequantised to F32;
* rms_norm (model.hpp:57-65): double sum of squares, float inverse,
  (x*inverse)*w as two float roundings;
* Matrix::multiply (quant.hpp:163-169): every weight dequantised to F32,
  dot products accumulated in double, cast to float;
* rotary (model.hpp:67-76): float angle pos/powf(theta, 2i/d), float cos/sin
  from the C oracle (same libm as the reference), split or interleaved pairs;
* fused_paged_attention (attention.hpp:57-83): GQA head h reads KV head
  h/(Hq/Hkv), scores q.k/sqrt(d) and softmax in double over all committed
  positions plus the current token;
* feedforward (model.hpp:115-126): SwiGLU with the overflow-safe sigmoid
  (C oracle), then the down projection;
* the LM head is output.weight when present, else the embedding (tied).

Position p's K/V are appended only after the whole token succeeds, exactly
as PagedModelExecutor::decode does.
"""

from __future__ import annotations

import numpy as np

from . import oracle as O
from tvara_b200.gguf import GGUFFile


class OracleModel:
    def __init__(self, path, max_positions: int | None = None, kv_quant: bool = False):
        # kv_quant: K and V rows pass through the int8 format of TVARA_KV_I8
        # pools (oracle/kvquant.py) before they are attended, as they are stored
        self.kv_quant = kv_quant
        f = GGUFFile(path)
        md = f.metadata
        self.vocab = len(md["tokenizer.ggml.tokens"])
        self.hidden = int(md["llama.embedding_length"])
        self.ffn = int(md["llama.feed_forward_length"])
        self.layers = int(md["llama.block_count"])
        self.heads = int(md["llama.attention.head_count"])
        self.kv_heads = int(md["llama.attention.head_count_kv"])
        self.context = int(md["llama.context_length"])
        self.eps = np.float32(md.get("llama.attention.layer_norm_rms_epsilon", 1e-6))
        self.theta = np.float32(md.get("llama.rope.freq_base", 10000.0))
        self.interleaved = md.get("tvara.rope.layout", "interleaved") == "interleaved"
        self.dim = self.hidden // self.heads
        self.kv_width = self.dim * self.kv_heads

        def mat(name):
            kind, shape = f.kind(name), f.shape(name)
            return O.dequantize(kind, f.raw(name), int(np.prod(shape))).reshape(shape)

        self.embedding = mat("token_embd.weight")
        self.output = mat("output.weight") if "output.weight" in f.tensors else self.embedding
        self.final_norm = mat("output_norm.weight")
        self.blocks = []
        for i in range(self.layers):
            p = f"blk.{i}."
            self.blocks.append({k: mat(p + k + ".weight") for k in (
                "attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up",
                "ffn_down")})
        self._f64 = {}
        n = max_positions or self.context
        self.cos, self.sin = O.rope_table(n, self.dim, float(self.theta))

    # ------------------------------------------------------------ primitives
    def matvec(self, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        key = id(w)
        w64 = self._f64.get(key)
        if w64 is None:
            w64 = self._f64[key] = w.astype(np.float64)
        return (w64 @ x.astype(np.float64)).astype(np.float32)

    def rms_norm(self, x, w):
        s = float(np.sum(x.astype(np.float64) ** 2))
        inv = np.float32(1.0 / np.sqrt(s / x.size + np.float64(self.eps)))
        return (x * inv).astype(np.float32) * w

    def rotary(self, x: np.ndarray, heads: int, pos: int) -> np.ndarray:
        d, half = self.dim, self.dim // 2
        v = x.reshape(heads, d).copy()
        c, s = self.cos[pos], self.sin[pos]
        if self.interleaved:
            a, b = v[:, 0::2].copy(), v[:, 1::2].copy()
            v[:, 0::2] = a * c - b * s
            v[:, 1::2] = b * c + a * s
        else:
            a, b = v[:, :half].copy(), v[:, half:].copy()
            v[:, :half] = a * c - b * s
            v[:, half:] = b * c + a * s
        return v.reshape(-1)

    def attention(self, q, keys, values):
        """keys/values: [positions, kv_width] float32 (committed + current)."""
        d, g = self.dim, self.heads // self.kv_heads
        out = np.empty(self.hidden, np.float32)
        k64 = keys.astype(np.float64).reshape(len(keys), self.kv_heads, d)
        v64 = values.astype(np.float64).reshape(len(values), self.kv_heads, d)
        q64 = q.astype(np.float64).reshape(self.heads, d)
        for h in range(self.heads):
            kh = h // g
            scores = (k64[:, kh, :] @ q64[h]) / np.sqrt(np.float64(d))
            w = np.exp(scores - scores.max())
            out[h * d:(h + 1) * d] = ((w @ v64[:, kh, :]) / w.sum()).astype(np.float32)
        return out

    def swiglu(self, gate, up):
        g = np.ascontiguousarray(gate, np.float32).copy()
        O.lib().orc_swiglu(g, np.ascontiguousarray(up, np.float32), g.size)
        return g

    # -------------------------------------------------------------- executor
    def new_state(self):
        return {"length": 0, "k": [[] for _ in range(self.layers)], "v": [[] for _ in range(self.layers)]}

    def fork(self, state):
        return {"length": state["length"], "k": [list(x) for x in state["k"]], "v": [list(x) for x in state["v"]]}

    def truncate(self, state, length):
        state["length"] = length
        for i in range(self.layers):
            state["k"][i] = state["k"][i][:length]
            state["v"][i] = state["v"][i][:length]

    def decode(self, state, token: int) -> np.ndarray:
        pos = state["length"]
        if token >= self.vocab or pos >= self.context:
            raise ValueError("paged decode exceeds token/context limits")
        x = self.embedding[token].astype(np.float32).copy()
        new_k, new_v = [], []
        for i, b in enumerate(self.blocks):
            xn = self.rms_norm(x, b["attn_norm"])
            q = self.rotary(self.matvec(b["attn_q"], xn), self.heads, pos)
            k = self.rotary(self.matvec(b["attn_k"], xn), self.kv_heads, pos)
            v = self.matvec(b["attn_v"], xn)
            if self.kv_quant:
                from oracle import kvquant
                k = kvquant.roundtrip(k.reshape(self.kv_heads, self.dim)).reshape(-1)
                v = kvquant.roundtrip(v.reshape(self.kv_heads, self.dim)).reshape(-1)
            keys = np.array(state["k"][i] + [k], np.float32)
            values = np.array(state["v"][i] + [v], np.float32)
            att = self.attention(q, keys, values)
            x = (x + self.matvec(b["attn_output"], att)).astype(np.float32)
            xn = self.rms_norm(x, b["ffn_norm"])
            ff = self.swiglu(self.matvec(b["ffn_gate"], xn), self.matvec(b["ffn_up"], xn))
            x = (x + self.matvec(b["ffn_down"], ff)).astype(np.float32)
            new_k.append(k)
            new_v.append(v)
        logits = self.matvec(self.output, self.rms_norm(x, self.final_norm))
        for i in range(self.layers):
            state["k"][i].append(new_k[i])
            state["v"][i].append(new_v[i])
        state["length"] = pos + 1
        return logits

    def forward(self, tokens) -> np.ndarray:
        st = self.new_state()
        return np.stack([self.decode(st, int(t)) for t in tokens])

    def greedy(self, prompt, steps: int) -> list[int]:
        st = self.new_state()
        logits = None
        for t in prompt:
            logits = self.decode(st, int(t))
        out = []
        for i in range(steps):
            tok = int(np.argmax(logits))
            out.append(tok)
            if i + 1 < steps:
                logits = self.decode(st, tok)
        return out


class RefEngine:
    """The reference engine itself through its C ABI (oracle/_ref), for
    pinning OracleModel and as the timed CPU baseline."""

    def __init__(self, path, max_blocks=256, block_tokens=16):
        import ctypes as C
        L = O.ref_capi()
        if L is None:
            raise FileNotFoundError("reference library not built")
        L.tvara_model_open.argtypes = [C.c_char_p, C.c_size_t, C.c_size_t]
        L.tvara_model_open.restype = C.c_void_p
        L.tvara_model_close.argtypes = [C.c_void_p]
        L.tvara_model_vocab_size.argtypes = [C.c_void_p]
        L.tvara_model_vocab_size.restype = C.c_size_t
        L.tvara_last_error.restype = C.c_char_p
        L.tvara_sequence_create.argtypes = [C.c_void_p]
        L.tvara_sequence_create.restype = C.c_uint64
        L.tvara_sequence_decode.argtypes = [C.c_void_p, C.c_uint64, C.c_uint32, O.f32p, C.c_size_t]
        L.tvara_sequence_drop.argtypes = [C.c_void_p, C.c_uint64]
        L.tvara_model_metadata.argtypes = [C.c_void_p]
        L.tvara_model_metadata.restype = C.c_char_p
        self.L = L
        self.h = L.tvara_model_open(str(path).encode(), max_blocks, block_tokens)
        if not self.h:
            raise RuntimeError(L.tvara_last_error().decode())
        self.vocab = L.tvara_model_vocab_size(self.h)

    def close(self):
        if self.h:
            self.L.tvara_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def create(self):
        return self.L.tvara_sequence_create(self.h)

    def drop(self, seq):
        self.L.tvara_sequence_drop(self.h, seq)

    def decode(self, seq, token):
        out = np.empty(self.vocab, np.float32)
        if self.L.tvara_sequence_decode(self.h, seq, token, out, self.vocab):
            raise RuntimeError(self.L.tvara_last_error().decode())
        return out

    def forward(self, tokens):
        s = self.create()
        try:
            return np.stack([self.decode(s, int(t)) for t in tokens])
        finally:
            self.drop(s)


class BatchOracle(OracleModel):
    """The same executor math for a ragged batch of sequences in one call, with
    the projections as float64 matrix products over all rows (each output is
    still a double-accumulated dot product cast to F32, as Matrix::multiply
    computes it; only the summation order differs) so that steps of hundreds
    of rows at 8B widths finish in seconds.

    ``step(batch)``: each entry of ``batch`` is a dict with ``tokens`` (the
    positions this step appends), ``start`` (positions already in the
    sequence) and ``history(layer) -> (keys, values)``, the sequence's
    committed K and V rows of that layer, [start, kv_heads*head_dim] F32.
    Returns the logits of every appended position, in batch order."""

    CHUNK = 8192  # weight rows converted to float64 at a time

    def mm(self, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        x64 = x.astype(np.float64)
        out = np.empty((x.shape[0], w.shape[0]), np.float32)
        for r in range(0, w.shape[0], self.CHUNK):
            out[:, r:r + self.CHUNK] = (x64 @ w[r:r + self.CHUNK].astype(np.float64).T).astype(np.float32)
        return out

    def rms_rows(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        s = np.sum(x.astype(np.float64) ** 2, axis=1)
        inv = (1.0 / np.sqrt(s / x.shape[1] + np.float64(self.eps))).astype(np.float32)
        return (x * inv[:, None]).astype(np.float32) * w

    def rotary_rows(self, x: np.ndarray, heads: int, pos: np.ndarray) -> np.ndarray:
        return np.stack([self.rotary(x[i], heads, int(p)) for i, p in enumerate(pos)])

    def attend(self, q: np.ndarray, keys: np.ndarray, values: np.ndarray) -> np.ndarray:
        """One query row over [positions, kv_width] keys/values (attention.hpp
        math in double, all heads at once)."""
        d, g, hk = self.dim, self.heads // self.kv_heads, self.kv_heads
        k64 = keys.astype(np.float64).reshape(len(keys), hk, d)
        v64 = values.astype(np.float64).reshape(len(values), hk, d)
        q64 = q.astype(np.float64).reshape(hk, g, d)
        scores = np.einsum("phd,hgd->hgp", k64, q64) / np.sqrt(np.float64(d))
        w = np.exp(scores - scores.max(axis=2, keepdims=True))
        out = np.einsum("hgp,phd->hgd", w, v64) / w.sum(axis=2)[..., None]
        return out.astype(np.float32).reshape(-1)

    def step(self, batch, kv_round=None) -> np.ndarray:
        """kv_round: optional function applied to the step's new K and V rows
        before they are attended (e.g. rounding to the pool's F16)."""
        rows = [(i, j) for i, e in enumerate(batch) for j in range(len(e["tokens"]))]
        tokens = np.array([batch[i]["tokens"][j] for i, j in rows], np.int64)
        pos = np.array([batch[i]["start"] + j for i, j in rows], np.int64)
        if np.any(tokens >= self.vocab) or np.any(pos >= self.context):
            raise ValueError("paged decode exceeds token/context limits")
        first = np.cumsum([0] + [len(e["tokens"]) for e in batch])
        x = self.embedding[tokens].astype(np.float32)
        for layer, b in enumerate(self.blocks):
            xn = self.rms_rows(x, b["attn_norm"])
            q = self.rotary_rows(self.mm(b["attn_q"], xn), self.heads, pos)
            k = self.rotary_rows(self.mm(b["attn_k"], xn), self.kv_heads, pos)
            v = self.mm(b["attn_v"], xn)
            if kv_round is not None:
                k, v = kv_round(k), kv_round(v)
            att = np.empty((len(rows), self.hidden), np.float32)
            for i, e in enumerate(batch):
                hk, hv = e["history"](layer)
                keys = np.concatenate([hk, k[first[i]:first[i + 1]]])
                values = np.concatenate([hv, v[first[i]:first[i + 1]]])
                for j in range(len(e["tokens"])):
                    visible = e["start"] + j + 1
                    att[first[i] + j] = self.attend(q[first[i] + j], keys[:visible], values[:visible])
            x = (x + self.mm(b["attn_output"], att)).astype(np.float32)
            xn = self.rms_rows(x, b["ffn_norm"])
            ff = self.swiglu(self.mm(b["ffn_gate"], xn), self.mm(b["ffn_up"], xn))
            x = (x + self.mm(b["ffn_down"], ff)).astype(np.float32)
        return self.mm(self.output, self.rms_rows(x, self.final_norm))
