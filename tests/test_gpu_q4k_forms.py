"""The packed Q4_K tensor-core kernel in each of its selectable forms.

The library reads TVARA_Q4K_A once per process (default: per launch, the
tensor-memory or the shared-memory form, whichever its tile plans make
faster; "tmem", "smem", "pair" force the one-CTA tensor-memory form, the
shared-memory form, the cta_group::2 CTA-pair kernel), so each forced form
reruns the parity tests of the tensor-core and narrow-row projections in a
child process: partial row tiles, several token tiles, split K, one to
sixteen 256-element blocks, every result within the oracle tolerance."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("form", ["tmem", "smem", "pair"])
def test_q4k_form_matches_oracle(form):
    env = dict(os.environ, TVARA_Q4K_A=form)
    res = subprocess.run(
        [sys.executable, "-m", "pytest", "tests/test_gpu_kernels.py", "-q", "-p", "no:cacheprovider", "-k",
         "(tensor_core_matmul and 12) or narrow_q4k or standalone_config_shape"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]
    assert " passed" in res.stdout
