"""Benchmark config 3 at its own sizes, on a B200, through the C ABI: the W8A8 GEMM over
M in {1, 16, 8192} x (K, N) in {(2048, 8192), (8192, 2048), (2048, 2048), (768, 262144)} with data
as in config 0 (N(0,1) activations with four outlier channels x20 quantised per token, N(0,0.02)
weights quantised per row). Bar: bit-exact to the reference fold. At M = 8192 the CPU check covers
a sample of rows (the first, the last, both neighbours of every 128-row tile boundary, random
ones): rows are independent in a GEMM, so a wrong tile shows in its sampled rows.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SWEEP_KN = [(2048, 8192), (8192, 2048), (2048, 2048), (768, 262144)]


@pytest.fixture(scope="module")
def weights(syn):
    cache = {}

    def get(K, N):
        if (K, N) not in cache:
            cache.clear()
            rng = np.random.default_rng(0xE2C0DE + 3 + K + N)
            w = np.empty((N, K), np.int8)
            s = np.empty(N, np.float32)
            for r0 in range(0, N, 65536):  # quantise in slices: the fp32 weight of N = 262144 is 0.8 GB
                r1 = min(N, r0 + 65536)
                w[r0:r1], s[r0:r1] = syn.quantize_weight_rows(
                    rng.standard_normal((r1 - r0, K), dtype=np.float32) * np.float32(0.02))
            cache[(K, N)] = (w, s)
        return cache[(K, N)]

    return get


@pytest.mark.parametrize("M", [1, 16, 8192])
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_config3_gemm_bitexact(e2c, of, syn, torch_cuda, weights, M, K, N):
    torch = torch_cuda
    w, ws = weights(K, N)
    rng = np.random.default_rng(M + K + N)
    x = syn.activations(rng, M, K)
    q, s = e2c.quantize_rows(torch.from_numpy(x).cuda(), K)
    W = e2c.Weight(w=w, scale=ws)
    y = e2c.i8_gemm(W, q, s, K)
    e2c.check()
    if M <= 16:
        rows = np.arange(M)
    else:
        edges = np.arange(128, M, 128)
        rows = np.unique(np.concatenate([[0, M - 1], edges - 1, edges, rng.integers(0, M, 16)]))
        if N > 100000:
            rows = np.unique(np.concatenate([rows[:: max(1, len(rows) // 40)], [M - 1]]))
    qh, sh = q.cpu().numpy()[rows], s.cpu().numpy()[rows]
    eq, es = of.quantize_signed(np.ascontiguousarray(x[rows]), K)
    assert np.array_equal(qh, eq) and np.array_equal(sh.view(np.int32), es.view(np.int32))
    want = of.gemm_plain(eq, es, w, ws, K)
    got = y[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    diff = got.view(np.int32) != want.view(np.int32)
    assert not diff.any(), f"{int(diff.sum())} of {diff.size} sampled outputs differ; max abs {np.abs(got - want).max()}"
    W.free()
