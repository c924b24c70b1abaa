import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a library")
    config.addinivalue_line("markers", "slow: full-size (8B-shape) cases")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.device_count() > 0
    except Exception:
        return False


HAS_GPU = _has_gpu()


def bits_equal(a, b) -> bool:
    """Bit-for-bit equality of two float32 arrays, except that any NaN
    matches any NaN: x86 SSE propagates an operand's NaN payload through
    a product, the GPU returns its canonical NaN, and the reference's
    decoder does produce NaNs for NaN/inf fp16 scales."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.shape != b.shape:
        return False
    same = a.view(np.uint32) == b.view(np.uint32)
    return bool(np.all(same | (np.isnan(a) & np.isnan(b))))


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_port():
    import oracle
    oracle.build(ref=False)
    return oracle.get("port")


@pytest.fixture(scope="session")
def oracle_ref():
    import oracle
    if not oracle.available("ref"):
        try:
            oracle.build(ref=True)
        except Exception:
            pass
    if not oracle.available("ref"):
        pytest.skip("reference engine (oracle/_ref) not built here")
    return oracle.get("ref")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        p = GOLDEN / name
        if p.suffix == ".npz":
            return dict(np.load(p))
        if p.suffix == ".json":
            import json
            return json.loads(p.read_text())
        return p.read_bytes()
    return load


@pytest.fixture(scope="session")
def eng():
    from distcomp_b200 import engine
    engine.lib()
    return engine


_models = {}


@pytest.fixture(scope="session")
def model_buf():
    """Seeded synthetic GGUF images, cached per (spec, seed)."""
    from distcomp_b200 import synth

    def get(key, seed=0, **over):
        k = (key, seed, tuple(sorted(over.items())))
        if k not in _models:
            _models[k] = synth.build_model(synth.spec(key, **over), seed=seed)
        return _models[k]
    return get
