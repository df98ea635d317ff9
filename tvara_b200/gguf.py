"""GGUF writing and block quantisation for synthetic Llama models.

The engine reads the GGUF subset the reference engine reads
(core/include/tvara/gguf.hpp:138-207, gguf_model.hpp:68-107): little-endian
v3 files, metadata scalars/strings/arrays, and tensors of type F32 (0),
F16 (1), Q4_0 (2), Q8_0 (8) and Q4_K (12).  This module writes such files
from numpy arrays so tests and benchmarks can build seeded models of any
shape.  Tensor dimensions are written innermost first, so a matrix with
``out`` rows of ``in`` inputs is stored with dims ``[in, out]``
(model.hpp:155-160 reads them back the same way).
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

F32, F16, Q4_0, Q8_0, Q4_K = 0, 1, 2, 8, 12
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144)}
TYPE_NAMES = {"f32": F32, "f16": F16, "q4_0": Q4_0, "q8_0": Q8_0, "q4_k": Q4_K}


def row_bytes(kind: int, cols: int) -> int:
    elems, width = BLOCK[kind]
    if cols % elems:
        raise ValueError(f"row width {cols} is not a multiple of {elems}")
    return cols // elems * width


# --------------------------------------------------------------------- quantisers
def quantize_q8_0(x: np.ndarray) -> bytes:
    """Q8_0 blocks: fp16 d = max|x|/127, int8 q = round(x/d) (the reference's
    own fixture writer uses the same rule, tools/make_api_fixture.py:128-138)."""
    blocks = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    d = (np.abs(blocks).max(axis=1) / 127).astype(np.float16)
    d32 = d.astype(np.float32)
    safe = np.where(d32 == 0, 1, d32)
    q = np.where(d32[:, None] == 0, 0, np.clip(np.round(blocks / safe[:, None]), -127, 127)).astype(np.int8)
    out = np.empty((blocks.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_0(x: np.ndarray) -> bytes:
    """Q4_0 blocks: fp16 d with value d*(q-8); element i in the low nibble of
    byte i, element i+16 in its high nibble (quant.hpp:51-61)."""
    blocks = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.abs(blocks).argmax(axis=1)
    peak = blocks[np.arange(blocks.shape[0]), idx]
    d = (peak / -8).astype(np.float16)
    d32 = d.astype(np.float32)
    safe = np.where(d32 == 0, 1, d32)
    q = np.where(d32[:, None] == 0, 8, np.clip(np.round(blocks / safe[:, None] + 8), 0, 15)).astype(np.uint8)
    out = np.empty((blocks.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.tobytes()


def pack_q4k_scales(scales: np.ndarray, mins: np.ndarray) -> np.ndarray:
    """Pack 8 six-bit scales and mins per block into the 12-byte field the
    reference decodes with q4k_scale_min (quant.hpp:63-68); the packing is the
    inverse that tests/core/test_quant.cpp:39-47 uses.  Arrays are [n, 8]."""
    s = np.asarray(scales, dtype=np.uint32) & 63
    m = np.asarray(mins, dtype=np.uint32) & 63
    enc = np.zeros((s.shape[0], 12), dtype=np.uint32)
    enc[:, 0:4] = s[:, 0:4]
    enc[:, 4:8] = m[:, 0:4]
    enc[:, 8:12] = (s[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)
    enc[:, 0:4] |= (s[:, 4:8] >> 4) << 6
    enc[:, 4:8] |= (m[:, 4:8] >> 4) << 6
    return enc.astype(np.uint8)


def quantize_q4_k(x: np.ndarray) -> bytes:
    """Q4_K super-blocks of 256: per 32-group an affine 4-bit code, the group
    scale and min quantised to 6 bits against fp16 d and dmin; the value is
    d*sc*q - dmin*m (quant.hpp:70-84)."""
    blocks = np.asarray(x, dtype=np.float32).reshape(-1, 8, 32)
    n = blocks.shape[0]
    lo = np.minimum(blocks.min(axis=2), 0)
    hi = blocks.max(axis=2)
    scale = (hi - lo) / 15
    mn = -lo
    d = (scale.max(axis=1) / 63).astype(np.float16)
    dmin = (mn.max(axis=1) / 63).astype(np.float16)
    d32, m32 = d.astype(np.float32), dmin.astype(np.float32)
    sc = np.clip(np.round(scale / np.where(d32 == 0, 1, d32)[:, None]), 0, 63).astype(np.uint32)
    mm = np.clip(np.round(mn / np.where(m32 == 0, 1, m32)[:, None]), 0, 63).astype(np.uint32)
    step = d32[:, None] * sc
    offset = m32[:, None] * mm
    q = np.where(step[:, :, None] == 0, 0,
                 np.clip(np.round((blocks + offset[:, :, None]) / np.where(step == 0, 1, step)[:, :, None]), 0, 15))
    q = q.astype(np.uint8)
    out = np.empty((n, 144), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = pack_q4k_scales(sc, mm)
    # byte 16 + p*32 + i holds group 2p (low nibble) and 2p+1 (high nibble)
    out[:, 16:] = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(n, 128)
    return out.tobytes()


def encode(kind: int, x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, dtype=np.float32)
    if kind == F32:
        return x.astype("<f4").tobytes()
    if kind == F16:
        return x.astype("<f2").tobytes()
    if kind == Q8_0:
        return quantize_q8_0(x)
    if kind == Q4_0:
        return quantize_q4_0(x)
    if kind == Q4_K:
        return quantize_q4_k(x)
    raise ValueError(f"unsupported tensor type {kind}")


# ------------------------------------------------------------- random packed blocks
def random_blocks(kind: int, rows: int, cols: int, rng: np.random.Generator,
                  d_range=(0.001, 0.05), dmin_range=None) -> bytes:
    """Packed blocks with uniformly random codes: fp16 d (and dmin) ~ U(d_range),
    Q4_K 6-bit scales/mins ~ U(0..63), nibbles ~ U(0..15), Q8_0 int8 ~
    U(-127..127).  Generation is byte-level so multi-GB tensors stay cheap."""
    elems, width = BLOCK[kind]
    nblocks = rows * (cols // elems)
    raw = np.frombuffer(rng.bytes(nblocks * width), dtype=np.uint8).reshape(nblocks, width).copy()
    if kind in (F32, F16):
        raise ValueError("random_blocks is for quantised types")
    d = rng.uniform(*d_range, size=nblocks).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    if kind == Q8_0:
        q = raw[:, 2:].view(np.int8)
        q[q == -128] = -127
    if kind == Q4_K:
        dm = rng.uniform(*(dmin_range or d_range), size=nblocks).astype(np.float16)
        raw[:, 2:4] = dm.view(np.uint8).reshape(-1, 2)
    return raw.tobytes()


# ------------------------------------------------------------------------ writer
def _string(value: str) -> bytes:
    data = value.encode("utf-8")
    return struct.pack("<Q", len(data)) + data


_SCALAR = {"u32": (4, "<I"), "i32": (5, "<i"), "f32": (6, "<f"), "bool": (7, "<B"),
           "u64": (10, "<Q"), "i64": (11, "<q"), "f64": (12, "<d")}


def _value(kind: str, value) -> tuple[int, bytes]:
    if kind == "str":
        return 8, _string(value)
    if kind.startswith("arr_"):
        inner = kind[4:]
        if inner == "str":
            return 9, struct.pack("<IQ", 8, len(value)) + b"".join(_string(v) for v in value)
        code, fmt = _SCALAR[inner]
        return 9, struct.pack("<IQ", code, len(value)) + b"".join(struct.pack(fmt, v) for v in value)
    code, fmt = _SCALAR[kind]
    return code, struct.pack(fmt, value)


def write_gguf(path, metadata: list[tuple[str, str, object]], tensors: list[tuple[str, int, tuple, bytes]],
               alignment: int = 32) -> Path:
    """Write a GGUF v3 file.  metadata entries are (key, kind, value) with kind
    one of str, u32, i32, f32, bool, u64, i64, f64, arr_<kind>; tensors are
    (name, type, shape outermost-first, payload bytes)."""
    path = Path(path)
    header = struct.pack("<4sIQQ", b"GGUF", 3, len(tensors), len(metadata))
    for key, kind, value in metadata:
        code, data = _value(kind, value)
        header += _string(key) + struct.pack("<I", code) + data
    offsets, offset = [], 0
    for name, kind, shape, payload in tensors:
        offset += (-offset) % alignment
        offsets.append(offset)
        offset += len(payload)
    infos = b""
    for (name, kind, shape, payload), off in zip(tensors, offsets):
        infos += _string(name) + struct.pack("<I", len(shape))
        infos += b"".join(struct.pack("<Q", d) for d in shape[::-1]) + struct.pack("<IQ", kind, off)
    head = header + infos
    head += b"\x00" * ((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        pos = 0
        for (name, kind, shape, payload), off in zip(tensors, offsets):
            f.write(b"\x00" * (off - pos))
            f.write(payload)
            pos = off + len(payload)
    return path


# ------------------------------------------------------------------- Llama models
LLAMA_CONFIGS = {
    # tiny, SmolLM2-135M shape, Llama-3-8B shape.
    "tiny": dict(vocab=512, hidden=256, layers=4, heads=8, kv_heads=2, ffn=688, eps=1e-5,
                 theta=10000.0, rope="split", context=2048, tied=True,
                 types=dict(default=Q8_0, ffn_down=F32, norm=F32, embd=Q8_0)),
    "smollm2": dict(vocab=49152, hidden=576, layers=30, heads=9, kv_heads=3, ffn=1536, eps=1e-5,
                    theta=100000.0, rope="split", context=8192, tied=True,
                    types=dict(default=Q8_0, norm=F32, embd=Q8_0)),
    "llama8b": dict(vocab=128256, hidden=4096, layers=32, heads=32, kv_heads=8, ffn=14336, eps=1e-5,
                    theta=500000.0, rope="split", context=8192, tied=False,
                    types=dict(default=Q4_K, norm=F32, embd=Q8_0, output=Q8_0)),
}


def tensor_plan(cfg: dict) -> list[tuple[str, tuple, int]]:
    """(name, shape, type) in the order weights are drawn."""
    t = cfg["types"]
    hidden, ffn, kv = cfg["hidden"], cfg["ffn"], cfg["hidden"] // cfg["heads"] * cfg["kv_heads"]
    plan = [("token_embd.weight", (cfg["vocab"], hidden), t.get("embd", t["default"]))]
    if not cfg.get("tied", True):
        plan.append(("output.weight", (cfg["vocab"], hidden), t.get("output", t["default"])))
    plan.append(("output_norm.weight", (hidden,), t.get("norm", F32)))
    for i in range(cfg["layers"]):
        p = f"blk.{i}."
        plan += [
            (p + "attn_norm.weight", (hidden,), t.get("norm", F32)),
            (p + "ffn_norm.weight", (hidden,), t.get("norm", F32)),
            (p + "attn_q.weight", (hidden, hidden), t.get("attn_q", t["default"])),
            (p + "attn_k.weight", (kv, hidden), t.get("attn_k", t["default"])),
            (p + "attn_v.weight", (kv, hidden), t.get("attn_v", t["default"])),
            (p + "attn_output.weight", (hidden, hidden), t.get("attn_output", t["default"])),
            (p + "ffn_gate.weight", (ffn, hidden), t.get("ffn_gate", t["default"])),
            (p + "ffn_up.weight", (ffn, hidden), t.get("ffn_up", t["default"])),
            (p + "ffn_down.weight", (hidden, ffn), t.get("ffn_down", t["default"])),
        ]
    return plan


def llama_metadata(cfg: dict) -> list:
    meta = [
        ("general.architecture", "str", "llama"),
        ("tvara.rope.layout", "str", cfg.get("rope", "split")),
        ("llama.attention.layer_norm_rms_epsilon", "f32", cfg["eps"]),
        ("llama.rope.freq_base", "f32", cfg["theta"]),
        ("llama.embedding_length", "u32", cfg["hidden"]),
        ("llama.feed_forward_length", "u32", cfg["ffn"]),
        ("llama.block_count", "u32", cfg["layers"]),
        ("llama.attention.head_count", "u32", cfg["heads"]),
        ("llama.attention.head_count_kv", "u32", cfg["kv_heads"]),
        ("llama.context_length", "u32", cfg["context"]),
        ("tokenizer.ggml.model", "str", "synthetic"),
        ("tokenizer.ggml.tokens", "arr_str", [f"t{i}" for i in range(cfg["vocab"])]),
    ]
    return meta + list(cfg.get("extra_metadata", []))


def make_llama(path, cfg: dict | str, seed: int = 0, std: float = 0.02, random_packed: bool = False,
               norm_ones: bool = False) -> Path:
    """Write a seeded random-weight Llama GGUF.  Weights are N(0, std) floats
    quantised to each tensor's type; norms are 1 + N(0, 0.1) (or ones).  With
    random_packed, quantised tensors are instead random blocks scaled so that
    |w| is about `std` -- used for multi-GB models where quantising floats in
    numpy would dominate set-up time."""
    if isinstance(cfg, str):
        cfg = LLAMA_CONFIGS[cfg]
    rng = np.random.default_rng(seed)
    tensors = []
    for name, shape, kind in tensor_plan(cfg):
        if len(shape) == 1:
            w = np.ones(shape, np.float32) if norm_ones else (1 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
            tensors.append((name, kind, shape, encode(kind, w)))
        elif random_packed and kind in (Q4_0, Q8_0, Q4_K):
            # mean |w| of a random code is about d * E|q| (Q8_0: ~64, Q4_0: ~4,
            # Q4_K: d*sc*q ~ 31*7.5 against an offset dmin*m ~ 31); pick d so
            # typical magnitudes are ~std.
            if kind == Q8_0:
                dr = (std / 64 * 0.5, std / 64 * 1.5)
                payload = random_blocks(kind, shape[0], shape[1], rng, dr)
            elif kind == Q4_0:
                dr = (std / 4 * 0.5, std / 4 * 1.5)
                payload = random_blocks(kind, shape[0], shape[1], rng, dr)
            else:
                dr = (std / 232 * 0.5, std / 232 * 1.5)
                payload = random_blocks(kind, shape[0], shape[1], rng, dr, (dr[0] * 7.5, dr[1] * 7.5))
            tensors.append((name, kind, shape, payload))
        else:
            w = rng.normal(0, std, shape).astype(np.float32)
            tensors.append((name, kind, shape, encode(kind, w)))
    return write_gguf(path, llama_metadata(cfg), tensors)


def model_config(name: str, **overrides) -> dict:
    cfg = dict(LLAMA_CONFIGS[name])
    cfg["types"] = dict(cfg["types"])
    for k, v in overrides.items():
        if k == "types":
            cfg["types"].update(v)
        else:
            cfg[k] = v
    return cfg


# ------------------------------------------------------------------------ reader
class GGUFFile:
    """Minimal GGUF v2/v3 reader (metadata + tensor payload views), used by
    tests and tools; the engine itself parses files in C++."""

    def __init__(self, path):
        self.path = Path(path)
        self.data = np.memmap(self.path, dtype=np.uint8, mode="r")
        buf = memoryview(self.data)
        pos = 0

        def take(n):
            nonlocal pos
            if pos + n > len(buf):
                raise ValueError("truncated GGUF data")
            out = bytes(buf[pos:pos + n])
            pos += n
            return out

        def u(fmt):
            return struct.unpack(fmt, take(struct.calcsize(fmt)))[0]

        def string():
            return take(u("<Q")).decode("utf-8", errors="surrogateescape")

        scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}

        def value(kind):
            if kind == 8:
                return string()
            if kind == 9:
                inner, count = u("<I"), u("<Q")
                return [value(inner) for _ in range(count)]
            v = u(scalar[kind])
            return bool(v) if kind == 7 else v

        if take(4) != b"GGUF":
            raise ValueError("invalid GGUF magic")
        self.version = u("<I")
        n_tensors, n_meta = u("<Q"), u("<Q")
        self.metadata = {}
        for _ in range(n_meta):
            key = string()
            self.metadata[key] = value(u("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = string()
            rank = u("<I")
            dims = [u("<Q") for _ in range(rank)]
            kind, off = u("<I"), u("<Q")
            self.tensors[name] = (kind, tuple(dims[::-1]), off)
        align = int(self.metadata.get("general.alignment", 32))
        self.data_offset = pos + (-pos) % align

    def raw(self, name) -> np.ndarray:
        kind, shape, off = self.tensors[name]
        n = int(np.prod(shape))
        elems, width = BLOCK[kind]
        start = self.data_offset + off
        return np.asarray(self.data[start:start + n // elems * width])

    def kind(self, name) -> int:
        return self.tensors[name][0]

    def shape(self, name) -> tuple:
        return self.tensors[name][1]
