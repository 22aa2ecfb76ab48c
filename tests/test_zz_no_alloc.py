"""e2cuda_i8_linear_noalloc against the allocating entry points it stands in for.

The no-allocation entry point quantises into the library's fixed per-device array and runs the W8A8
GEMM from there; its result must equal e2cuda_quantize_rows followed by e2cuda_i8_gemm (caller
buffers) on the same input. Two calls in a row, with different inputs and row counts, check that
the second call does not read anything the first one left in the shared array. This file sorts last
so that it runs both alone in a fresh process and after every other GPU test.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _weight(e2c, syn, rng, N, K):
    q, s = syn.quantize_weight_rows(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    return e2c.Weight(w=q, scale=s)


def _allocating(e2c, W, x, ablk):
    qa, qs = e2c.quantize_rows(x, ablk)
    return e2c.i8_gemm(W, qa, qs, ablk)


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
        got, ref = y.cpu().numpy(), want.cpu().numpy()
        # the same kernels on the same bytes: equal up to fp32 rounding of the epilogue
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6 * float(np.abs(ref).max()))


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
    want = _allocating(e2c, W, xs, K)
    np.testing.assert_allclose(ys.cpu().numpy(), want.cpu().numpy(), rtol=1e-6,
                               atol=1e-6 * float(want.abs().max()))
