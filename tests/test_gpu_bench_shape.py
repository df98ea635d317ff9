"""Parity at the benchmarked shape: a 2-layer model with the Llama-3-8B
widths (hidden 4096, FFN 14336, 32/8 heads of 128, RoPE theta 5e5, Q4_K
projections, Q8_0 embedding and LM head over a 128256 vocabulary) runs one
ragged tvara_batch_step of 256 sequences -- one token each, 2..8 for sixteen
of them -- that share a 1000-position prefix through the radix cache
(copy-on-write of its partial tail block) and hold 64..1000 positions of their
own, so contexts reach ~2k and the projections run at ~300 rows with the
tile / split-K planner at 8B widths.  Every row's logits are checked against
the CPU oracle (oracle/parity.py): |d| <= 2e-3 + 1e-3 |want|, argmax equal
except on near-ties.

F32 KV (the reference's format) is checked against the reference's
arithmetic directly.  An F16 pool stores each new K/V row rounded to F16; at
these widths that storage alone moves logits by up to ~1e-2 from the F32
reference (the CPU oracle shows the same when it rounds the new rows), so the
F16 case is checked against the oracle with that rounding applied, within
twice the bound (oracle/parity.py F16_ATOL / F16_RTOL), and the distance to
the F32 reference is bounded separately."""

import numpy as np
import pytest

from oracle import parity
from tvara_b200 import gguf
from tvara_b200.native import NativeModel
from tests.conftest import make_model

pytestmark = pytest.mark.gpu

REQUESTS, PREFIX, SUFFIX, EXTRA = 256, 1000, (64, 1000), 16


@pytest.fixture(scope="module")
def llama8b_2l(model_dir):
    return make_model(model_dir, "llama8b_l2", gguf.model_config("llama8b", layers=2), seed=0, random_packed=True)


@pytest.mark.parametrize("kv", ["f16", "f32"])
def test_llama8b_widths_ragged_step_matches_oracle(llama8b_2l, kv):
    tpb = 16
    per_request = (PREFIX + SUFFIX[1] + 8 + tpb - 1) // tpb - PREFIX // tpb + 1
    blocks = REQUESTS * per_request + PREFIX // tpb + 8
    with NativeModel(llama8b_2l, max_blocks=blocks, block_tokens=tpb, kv_dtype=kv, max_step_tokens=2048) as m:
        case = parity.build_step(m, seed=21, requests=REQUESTS, prefix=PREFIX, suffix=SUFFIX, extra_rows=EXTRA)
        got, am = m.batch_step(case["seqs"], case["tokens"], all_logits=True, argmax=True)
        assert np.array_equal(am, np.argmax(got, axis=1))
        for s in case["seqs"]:
            m._drop_sequence(s)
        m.prefix_unpin(case["node"])
        m._drop_sequence(case["src"])
        m.kv_audit()
    assert got.shape == (sum(len(t) for t in case["tokens"]), 128256)
    f16 = (lambda a: a.astype(np.float16).astype(np.float32)) if kv == "f16" else None
    want = parity.oracle_rows(llama8b_2l, case, max_positions=PREFIX + SUFFIX[1] + 16, kv_round=f16)
    res = parity.compare(got, want) if kv == "f32" else parity.compare(got, want, parity.F16_ATOL, parity.F16_RTOL)
    assert res["ok"], res
    if kv == "f16":
        ref = parity.oracle_rows(llama8b_2l, case, max_positions=PREFIX + SUFFIX[1] + 16)
        assert np.abs(got - ref).max() <= 3e-2
