"""One process driving two GPUs in turn: every kernel's set-up (the shared-memory opt-in, the
resident-cluster counts, the SM count) is kept per device, so device 1's first launches get their
own set-up and device 0's later launches keep theirs. Each op runs on device 0, then device 1, then
device 0 again, and the three results must be bit-identical. Skipped with fewer than two GPUs."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ops(e2c, syn, torch, dev):
    """The results of the per-token persistent GEMM, the short-activation GEMM (split-K or
    streaming), the GEMM with the residual norms in its epilogue (a cluster kernel) and the
    attention, all on `dev`, as host arrays."""
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(11)
    D, N = 768, 2304
    w = rng.integers(-127, 128, size=(N, D), dtype=np.int8)
    ws = rng.uniform(1e-4, 0.02, size=N).astype(np.float32)
    W = e2c.Weight(w=w, scale=ws)
    out = []
    for M in (4096, 8):
        x = torch.from_numpy(rng.standard_normal((M, D)).astype(np.float32)).to(dev)
        qa, qs = e2c.quantize_rows(x, D)
        out.append(e2c.i8_gemm(W, qa, qs).cpu().numpy())
    # o_proj-shaped GEMM with the residual norms fused (clusters of D / 128 CTAs)
    M = 2048
    wo = rng.integers(-127, 128, size=(D, D), dtype=np.int8)
    wos = rng.uniform(1e-4, 0.02, size=D).astype(np.float32)
    Wo = e2c.Weight(w=wo, scale=wos)
    x = torch.from_numpy(rng.standard_normal((M, D)).astype(np.float32)).to(dev)
    qa, qs = e2c.quantize_rows(x, D)
    res = torch.from_numpy(rng.standard_normal((M, D)).astype(np.float32)).to(dev)
    g = torch.ones(D, device=dev)
    q8 = torch.zeros((M, D), dtype=torch.int8, device=dev)
    q8s = torch.zeros((M,), dtype=torch.float32, device=dev)
    a = e2c.gemm_args(Wo, qa, qs, M)
    a.epi, a.eps = e2c.EPI_NORMADD, 1e-6
    a.res, a.ldres, a.norm_g1, a.norm_g2 = res.data_ptr(), D, g.data_ptr(), g.data_ptr()
    a.q8, a.ldq, a.q8_scale = q8.data_ptr(), D, q8s.data_ptr()
    e2c.gemm_raw(a)
    e2c.check()
    out += [res.cpu().numpy(), q8.cpu().numpy(), q8s.cpu().numpy()]
    # attention: 2 sequences of 256 tokens, 3 heads of 256, one KV head
    B, S, H, Dh = 2, 256, 3, 256
    q = torch.from_numpy(rng.standard_normal((B * S, H * Dh)).astype(np.float32)).to(dev).to(torch.bfloat16)
    k = torch.from_numpy(rng.standard_normal((B * S, Dh)).astype(np.float32)).to(dev).to(torch.bfloat16)
    vt = torch.from_numpy(rng.standard_normal((B, Dh, S)).astype(np.float32)).to(dev).to(torch.bfloat16)
    out.append(e2c.attention(q, k, vt, None, B, S, H, 1.0 / 16).cpu().numpy())
    torch.cuda.synchronize(dev)
    return out


def test_two_devices_in_one_process(e2c, syn, torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU: the per-device set-up needs a second device to switch to")
    first = _ops(e2c, syn, torch, 0)
    other = _ops(e2c, syn, torch, 1)
    again = _ops(e2c, syn, torch, 0)
    torch.cuda.set_device(0)
    for i, (a, b, c) in enumerate(zip(first, other, again)):
        assert a.tobytes() == b.tobytes(), f"result {i} differs on device 1"
        assert a.tobytes() == c.tobytes(), f"result {i} differs on device 0 after device 1"
