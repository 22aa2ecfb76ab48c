"""The drop-in boundary without a GPU: libe2cuda.so loads, exports every function include/e2cuda.h
declares, the Python mirror binds exactly those, and the e2_q8w-compatible structures match the
reference's layout. No compute is called here."""
from __future__ import annotations

import ctypes as C
import re

import pytest


def declared_functions(header_text: str) -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", header_text, flags=re.S)
    return set(re.findall(r"\b(e2cuda_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol(e2c):
    names = declared_functions(e2c.HEADER.read_text())
    assert len(names) >= 20
    lib = C.CDLL(str(e2c.LIB_PATH))
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    bound = {n for n, _, _ in e2c.API}
    assert bound == names, f"python mirror out of sync: {sorted(bound ^ names)}"


def test_q8w_layout_matches_reference_struct(e2c, of):
    # e2cuda_q8w (include/e2cuda.h) == e2o_q8w == e2_q8w (e2.c src/int8.h:79-92)
    a, b = e2c.Q8W, of.Q8W
    assert C.sizeof(a) == C.sizeof(b)
    for (na, _), (nb, _) in zip(a._fields_, b._fields_):
        assert na == nb and getattr(a, na).offset == getattr(b, nb).offset


def test_no_cpu_fallback(e2c, monkeypatch):
    """Without a CUDA device the ops raise; there is no host path that could stand in for them."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(e2c.E2CudaError):
        e2c.quantize_rows(torch.zeros((4, 16)), 16)


def test_error_reporting_without_device(e2c):
    lib = e2c.lib()
    # argument validation happens before any device work: a bad call fails with a message
    assert lib.e2cuda_ffn_create(None, None, None, None, 1e-6, 16) is None
    assert "ffn_create" in e2c.last_error()


def test_gemm_args_layout_matches_the_library(e2c):
    """The launcher's argument struct (csrc/launch.h) and its ctypes mirror have the same size."""
    lib = C.CDLL(str(e2c.LIB_PATH))
    lib.e2c_gemm_args_size.restype = C.c_int
    assert lib.e2c_gemm_args_size() == C.sizeof(e2c.GemmArgs)
