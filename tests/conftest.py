"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on a CPU-only host.

``e2c`` is the product package (``e2.c_b200``, loaded by path because of the dot in its name);
``of`` is the CPU checker (``oracle/oracle_ffi.py``), used here only to compute expected values.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); run with -m gpu on a B200")


def load_e2c():
    if "e2c_b200" in sys.modules:
        return sys.modules["e2c_b200"]
    pkg = ROOT / "e2.c_b200"
    spec = importlib.util.spec_from_file_location("e2c_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["e2c_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def e2c():
    return load_e2c()


@pytest.fixture(scope="session")
def syn():
    load_e2c()
    import e2c_b200.synthetic as s

    return s


@pytest.fixture(scope="session")
def of():
    from oracle import oracle_ffi

    oracle_ffi.port()  # fail loudly if the checker was not built
    return oracle_ffi


@pytest.fixture(scope="session")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return torch


def cosine_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1) + 1e-300)


def tie_tolerant_bytes(got: np.ndarray, want: np.ndarray, pre_round: np.ndarray, band: float = 2e-3) -> None:
    """Quantised bytes after an fp32 epilogue (the reference's own rule in
    tests/test_gpu_ffn.c:112-118): equal, or one step apart where the pre-round value is within
    `band` of a .5 tie."""
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    near = np.abs(np.abs(pre_round - np.floor(pre_round)) - 0.5) < band
    bad = (d > 1) | ((d == 1) & ~near)
    assert not bad.any(), f"{int(bad.sum())} bytes differ beyond the tie rule (of {d.size}); max delta {int(d.max())}"


# ------------------------------------------------------------------------------ e2.c's own text tower
@pytest.fixture(scope="session")
def text_tensors():
    """The seeded random-init text-tower checkpoint (bf16 bit patterns by tensor name)."""
    load_e2c()
    import e2c_b200.text_model as tm

    return tm.random_tensors()


@pytest.fixture(scope="session")
def text_model_dir(tmp_path_factory, text_tensors):
    """<dir>/model.safetensors of text_tensors, as e2.c's loader reads it."""
    import e2c_b200.text_model as tm

    d = tmp_path_factory.mktemp("text_model")
    tm.write_safetensors(d / "model.safetensors", text_tensors)
    return d


@pytest.fixture(scope="session")
def ref_text(of, text_model_dir):
    """e2.c's own engine with the checkpoint loaded (one model per process, e2.c's rule)."""
    r = of.RefText()
    r.load(text_model_dir, text_model_dir / "text.e8cq")
    yield r
    r.free()
