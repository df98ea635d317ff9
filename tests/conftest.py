import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle as O
    return O.lib()


@pytest.fixture(scope="session")
def ref_shim():
    from oracle import oracle as O
    r = O.ref()
    if r is None:
        pytest.skip("reference not compiled here (oracle/_ref)")
    return r


@pytest.fixture(scope="session")
def capi():
    """The engine library (built in-tree); fails loudly when missing."""
    from tvara_b200 import load_library
    return load_library()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def make_model(model_dir, name, cfg, seed=0, **kw):
    from tvara_b200 import gguf
    path = model_dir / f"{name}.gguf"
    if not path.exists():
        gguf.make_llama(path, cfg, seed=seed, **kw)
    return path


@pytest.fixture(scope="session")
def tiny_path(model_dir):
    return make_model(model_dir, "tiny", "tiny", seed=0)
