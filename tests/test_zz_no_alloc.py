"""e2cuda_i8_linear_noalloc against the allocating entry points it stands in for.

The no-allocation entry point serves callers that cannot let a library allocate device memory (a
server whose allocator already holds its HBM budget, a latency-bound loop that must never meet
cudaMalloc's blocking and device-wide synchronisation, a host with a fixed device footprint). It
quantises into the library's fixed per-device array and runs the W8A8 GEMM from there; its result
must equal e2cuda_quantize_rows followed by e2cuda_i8_gemm (caller buffers) on the same input, bit
for bit, since the same kernels run on the same bytes. Two calls in a row, with different inputs
and row counts, check that the second call does not read anything the first one left in the shared
array. A fresh process checks that repeated calls leave the device's free memory unchanged.

This file sorts last so that it runs both alone in a fresh process and after every other GPU test.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _weight(e2c, syn, rng, N, K):
    q, s = syn.quantize_weight_rows(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    return e2c.Weight(w=q, scale=s)


def _allocating(e2c, W, x, ablk):
    qa, qs = e2c.quantize_rows(x, ablk)
    return e2c.i8_gemm(W, qa, qs, ablk)


def _same_bits(got, want):
    g, w = got.cpu().numpy(), want.cpu().numpy()
    assert g.shape == w.shape
    diff = g.view(np.int32) != w.view(np.int32)
    assert not diff.any(), f"{int(diff.sum())} of {diff.size} outputs differ from the allocating path"


@pytest.mark.parametrize("N,K,ablk", [(768, 768, None), (1152, 768, 128), (200, 1152, None)])
def test_noalloc_matches_allocating_path_twice(e2c, syn, torch_cuda, N, K, ablk):
    torch = torch_cuda
    rng = np.random.default_rng(0x0A110C + N + K)
    W = _weight(e2c, syn, rng, N, K)
    ablk_v = ablk or K
    for M in (1000, 333):  # the second call is smaller: stale rows of the first must not leak in
        x = torch.from_numpy(syn.activations(rng, M, K)).cuda()
        want = _allocating(e2c, W, x, ablk_v)
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        e2c.i8_linear_noalloc(W, x, y, ablk_v)
        e2c.check()
        _same_bits(y, want)


def test_noalloc_rejects_rows_beyond_the_scratch(e2c, syn, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    K = 768
    W = _weight(e2c, syn, rng, 256, K)
    m_fit = (e2c.NOALLOC_SCRATCH_BYTES - 512) // (K + 4)
    m_big = e2c.NOALLOC_SCRATCH_BYTES // K + 1
    x = torch.zeros((m_big, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((m_big, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(e2c.E2CudaError, match="maximum"):
        e2c.i8_linear_noalloc(W, x, y)
    # the largest row count that fits still runs, and agrees with the allocating path
    xs = torch.from_numpy(syn.activations(rng, m_fit, K)).cuda()
    ys = torch.empty((m_fit, 256), dtype=torch.float32, device="cuda")
    e2c.i8_linear_noalloc(W, xs, ys)
    _same_bits(ys, _allocating(e2c, W, xs, K))


def test_noalloc_refuses_a_capturing_stream(e2c, syn, torch_cuda):
    """The call synchronises its stream to read its status; on a capturing stream it returns an
    error before queuing anything, and the caller's capture stays valid."""
    torch = torch_cuda
    rng = np.random.default_rng(6)
    K = 768
    W = _weight(e2c, syn, rng, 128, K)
    x = torch.from_numpy(syn.activations(rng, 64, K)).cuda()
    y = torch.zeros((64, 128), dtype=torch.float32, device="cuda")
    e2c.i8_linear_noalloc(W, x, y)  # the first call on the device does the set-up, outside capture
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    refused = None
    with torch.cuda.graph(g, stream=s):
        try:
            e2c.i8_linear_noalloc(W, x, y, stream=s)
        except e2c.E2CudaError as ex:
            refused = str(ex)
        y.add_(1.0)  # the capture is still usable after the refusal
    assert refused is not None and "captured" in refused
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert bool((y == 1.0).all())


def test_noalloc_leaves_free_memory_unchanged_fresh_process(torch_cuda):
    """In a fresh process (no library state from earlier tests), repeated calls at several row
    counts and activation blocks leave the device's free memory where the first round left it."""
    r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "free-memory"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "free memory unchanged" in r.stdout, r.stdout[-2000:]


def _free_memory_check() -> int:
    import torch

    root = Path(__file__).resolve().parent
    sys.path.insert(0, str(root))
    from conftest import load_e2c

    e2c = load_e2c()
    import e2c_b200.synthetic as syn

    torch.cuda.set_device(0)
    rng = np.random.default_rng(11)
    K, N = 768, 1152
    W = _weight(e2c, syn, rng, N, K)
    cases = []
    for M, ablk in ((1, K), (16, K), (333, K), (1000, 128), (4096, K)):
        x = torch.from_numpy(syn.activations(rng, M, K)).cuda()
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        cases.append((x, y, ablk))
    torch.cuda.synchronize()
    for x, y, ablk in cases:  # first round: lazy module loading and the per-device set-up happen here
        e2c.i8_linear_noalloc(W, x, y, ablk)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for x, y, ablk in cases:
            e2c.i8_linear_noalloc(W, x, y, ablk)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    if free1 < free0:
        print(f"free memory dropped by {free0 - free1} bytes over {3 * len(cases)} calls")
        return 1
    print(f"free memory unchanged over {3 * len(cases)} calls ({free0} -> {free1} bytes)")
    return 0


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "free-memory":
        sys.exit(_free_memory_check())
