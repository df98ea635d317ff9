"""Regenerate the golden fixtures in this directory from the reference engine.

Run where oracle/_ref was built from a Tvara checkout
(``make -C oracle REFERENCE=/path/to/Tvara``, which also stages the
reference's Python package into oracle/_ref/python):

    python tests/golden/make_golden.py

Every model is rebuilt deterministically by tvara_b200.gguf.make_llama from
its seed, so only the reference's outputs are stored:

* tiny_q8.npz     -- BASELINE tiny config (Q8_0, F32 ffn_down, split RoPE):
                     64-token seeded prompt, 64 greedy tokens chosen by the
                     reference, and the reference's F32 logits at all 128
                     positions (teacher-forced on prompt + greedy tokens).
* tiny_mixed.npz  -- same shape with Q4_K / Q4_0 / F16 projections and
                     interleaved RoPE: 24 positions of logits.
* dequant.npz     -- random GGUF blocks of each type (including fp16 scale
                     bit patterns that are subnormal, inf and NaN) and the
                     reference's dequantised floats.
* sampling.npz    -- tokens from the reference's own NativeModel.iter_tokens
                     (python/tvara/native.py, over its C++ library in
                     oracle/_ref) on the tiny model: greedy with repetition /
                     frequency / presence penalties and an even-token
                     constraint, and seeded temperature / top-k / min-p /
                     top-p sampling with penalties.  Only this file:
                     ``python tests/golden/make_golden.py sampling``.
* quantized_kv.npz -- rows (zero, subnormal, tiny, large, exact .5 ties,
                     random) and the codes and scales of the reference's own
                     QuantizedKV.encode (python/tvara/quantized_kv.py).  Only
                     this file: ``python tests/golden/make_golden.py kv``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from tvara_b200 import gguf  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.model import RefEngine  # noqa: E402
from oracle.oracle import reference_module  # noqa: E402
from tests.golden.sampling_cases import SAMPLING_CASES, EvenTokens  # noqa: E402

TINY_PROMPT_SEED = 1
MIXED = dict(rope="interleaved", types=dict(attn_q=gguf.Q4_K, attn_k=gguf.Q4_0, attn_v=gguf.F16,
                                             ffn_gate=gguf.Q4_K, ffn_up=gguf.Q4_K, attn_output=gguf.Q4_0))


def tiny_prompt():
    return np.random.default_rng(TINY_PROMPT_SEED).integers(0, 512, 64).astype(np.int64)


def reference_greedy(engine, prompt, steps):
    s = engine.create()
    logits = [engine.decode(s, int(t)) for t in prompt]
    out = []
    for _ in range(steps):
        tok = int(np.argmax(logits[-1]))
        out.append(tok)
        logits.append(engine.decode(s, tok))
    engine.drop(s)
    return out, np.stack(logits[:len(prompt) + steps])


def random_blocks(rng, kind, n):
    elems, width = gguf.BLOCK[kind]
    raw = rng.integers(0, 256, size=(n, width), dtype=np.uint8)
    specials = np.array([0x0000, 0x0001, 0x03ff, 0x0400, 0x3c00, 0xbc00, 0x7bff, 0x7c00, 0xfc00, 0x7e00, 0x7c01,
                         0x8000, 0x8001], dtype=np.uint16)
    if kind in (gguf.Q8_0, gguf.Q4_0, gguf.Q4_K):
        d = rng.choice(specials, size=n)
        normal = rng.uniform(-1, 1, size=n).astype(np.float16).view(np.uint16)
        d = np.where(rng.random(n) < 0.5, normal, d).astype(np.uint16)
        raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return raw


def sampling_golden(tiny_path):
    import os
    RefNativeModel = reference_module("native").NativeModel
    lib = ROOT / "oracle" / "_ref" / "libtvara_capi.so"
    os.environ["TVARA_LIBRARY"] = str(lib)
    prompt = [int(t) for t in tiny_prompt()[:24]]
    out = {"prompt": np.array(prompt)}
    with RefNativeModel(str(tiny_path), library=str(lib)) as model:
        for name, case in SAMPLING_CASES.items():
            kw = dict(case)
            constraint = EvenTokens(model.vocab_size) if kw.pop("constraint", False) else None
            toks = list(model.iter_tokens(prompt, max_new_tokens=32, token_constraint=constraint, **kw))
            out[name] = np.array(toks)
    np.savez_compressed(HERE / "sampling.npz", **out)


def quantized_kv_golden():
    QuantizedKV = reference_module("quantized_kv").QuantizedKV
    rng = np.random.default_rng(4242)
    d = 64
    rows = [np.zeros(d, np.float32), np.full(d, 1e-44, np.float32), np.full(d, 1e-30, np.float32),
            (rng.standard_normal(d) * 3e38 / 4).astype(np.float32)]
    tie = np.zeros(d, np.float32)
    tie[0] = 127.0
    tie[1:] = np.arange(1, d, dtype=np.float32) + 0.5  # exact halves after dividing by a scale of 1
    rows.append(tie)
    rows += [(rng.standard_normal(d) * s).astype(np.float32) for s in (1e-3, 1.0, 30.0)]
    rows += [(rng.standard_normal(d) * rng.uniform(0.01, 10)).astype(np.float32) for _ in range(24)]
    rows = np.stack(rows)
    codes, scales = QuantizedKV.encode(rows)
    np.savez_compressed(HERE / "quantized_kv.npz", rows=rows, codes=codes, scales=scales)


def main():
    import tempfile
    if sys.argv[1:] == ["kv"]:
        quantized_kv_golden()
        print("wrote quantized_kv.npz")
        return
    if sys.argv[1:] == ["sampling"]:
        tmp = Path(tempfile.mkdtemp())
        sampling_golden(gguf.make_llama(tmp / "tiny.gguf", "tiny", seed=0))
        print("wrote sampling.npz")
        return
    tmp = Path(tempfile.mkdtemp())
    tiny = gguf.make_llama(tmp / "tiny.gguf", "tiny", seed=0)
    ref = RefEngine(tiny)
    prompt = tiny_prompt()
    greedy, logits = reference_greedy(ref, prompt, 64)
    np.savez_compressed(HERE / "tiny_q8.npz", prompt=prompt, greedy=np.array(greedy), logits=logits)

    cfg = gguf.model_config("tiny", **MIXED)
    mixed = gguf.make_llama(tmp / "mixed.gguf", cfg, seed=3)
    ref2 = RefEngine(mixed)
    toks = np.random.default_rng(2).integers(0, 512, 24)
    np.savez_compressed(HERE / "tiny_mixed.npz", tokens=toks, logits=ref2.forward(toks))

    rng = np.random.default_rng(2026)
    out = {}
    R = O.ref()
    for kind in (gguf.Q8_0, gguf.Q4_0, gguf.Q4_K, gguf.F16, gguf.F32):
        elems, width = gguf.BLOCK[kind]
        n = 64 if elems > 1 else 4096
        raw = random_blocks(rng, kind, n)
        vals = np.empty(n * elems, np.float32)
        assert R.ref_dequantize(kind, np.ascontiguousarray(raw.reshape(-1)), raw.size, vals, vals.size) == 0
        out[f"raw_{kind}"] = raw.reshape(-1)
        out[f"out_{kind}"] = vals.view(np.uint32)
    np.savez_compressed(HERE / "dequant.npz", **out)
    sampling_golden(tiny)
    quantized_kv_golden()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
