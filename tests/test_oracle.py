"""Pin the CPU port against the reference e2.c kernels compiled from their own sources
(oracle/_ref/, built by oracle/Makefile where the reference sources exist; skipped elsewhere, where
tests/test_golden.py covers the same ground from committed fixtures).

Coverage follows the reference's own tests: tests/test_scalar_kernels.c (chunked-vs-whole GEMM,
quantiser scales and bytes, column ranges, clipped outputs), tests/test_int8.c (every x86 backend,
outliers, tails), tests/test_gpu_ffn.c (FFN stages, tie rule).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import cosine_rows

pytestmark = pytest.mark.skipif(
    not __import__("oracle.oracle_ffi", fromlist=["x"]).ref_available(128),
    reason="reference builds absent (oracle/_ref); tests/test_golden.py pins the port instead")


def _x(syn, rng, M, K):
    x = syn.activations(rng, M, K) * rng.uniform(1e-3, 10, (M, 1)).astype(np.float32)
    x = np.ascontiguousarray(x, np.float32)
    x[0] = 0
    return x


@pytest.mark.parametrize("blk,M,K", [(128, 64, 768), (128, 33, 2048), (768, 40, 768), (1152, 17, 1152),
                                     (2048, 9, 2048), (8192, 3, 8192), (3072, 5, 3072), (256, 8, 1024)])
@pytest.mark.parametrize("fn", ["e2_quantize_blocks_avx512", "e2_quantize_blocks_scalar"])
def test_quantizer_bitexact_vs_reference(of, syn, blk, M, K, fn):
    rng = np.random.default_rng(blk + M + K)
    x = _x(syn, rng, M, K)
    x[min(2, M - 1), :blk] = 0
    lib = of.ref(blk)
    rq, rs = of.quantize_biased(x, blk, lib=lib, fn=fn)
    pq, ps = of.quantize_biased(x, blk)
    assert np.array_equal(rq, pq)
    assert np.array_equal(rs.view(np.int32), ps.view(np.int32))


def test_quantizer_clamp_and_simd_backends(of, syn):
    rng = np.random.default_rng(2)
    x = _x(syn, rng, 16, 512)
    lib = of.ref(128)
    pq, ps = of.quantize_biased(x, 128, -0.75, 0.75)
    rq, rs = of.quantize_biased(x, 128, -0.75, 0.75, lib=lib, fn="e2_quantize_blocks_avx512")
    assert np.array_equal(rq, pq) and np.array_equal(rs, ps)
    # the reference admits +-1 between its scalar and 256-bit quantisers (tests/test_scalar_kernels.c:221-233)
    for fn in ("e2_quantize_blocks_avx2", "e2_quantize_blocks_vnni"):
        q2, s2 = of.quantize_biased(x, 128, lib=lib, fn=fn)
        pq2, ps2 = of.quantize_biased(x, 128)
        assert np.abs(q2.astype(int) - pq2.astype(int)).max() <= 1
        np.testing.assert_allclose(s2, ps2, rtol=1e-6)


@pytest.mark.parametrize("blk,N,K", [(128, 40, 256), (128, 200, 768), (768, 64, 768), (2048, 24, 2048),
                                     (8192, 16, 8192), (1152, 8, 1152)])
def test_weight_quantiser_and_pack_vs_reference(of, syn, blk, N, K):
    rng = np.random.default_rng(N * K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[3] = 0
    lib = of.ref(blk)
    r, p = of.Weight(w, blk, lib), of.Weight(w, blk)
    assert np.array_equal(r.q.packed(), p.q.packed())
    assert np.array_equal(r.q.scales().view(np.int32), p.q.scales().view(np.int32))
    assert np.array_equal(r.q.bsums(), p.q.bsums())
    # and the numpy quantiser/packer the synthetic models and bench use
    pw = syn.PackedWeight(*syn.quantize_weight_rows(w), blk)
    assert np.array_equal(pw.packed, p.q.packed()) and np.array_equal(pw.bsq, p.q.bsums())
    assert np.array_equal(pw.scale_pad.view(np.int32), p.q.scales().view(np.int32))


@pytest.mark.parametrize("blk,M,N,K,n0,n1", [(128, 64, 512, 2048, 0, 512), (128, 15, 256, 512, 0, 256),
                                             (128, 4, 40, 384, 3, 29), (768, 512, 1152, 768, 0, 1152),
                                             (1152, 33, 96, 1152, 16, 80), (2048, 8, 64, 2048, 0, 64)])
@pytest.mark.parametrize("fn", ["e2_i8_gemm_avx512", "e2_i8_gemm_scalar", "e2_i8_gemm_avx2"])
def test_gemm_bitexact_vs_reference(of, syn, blk, M, N, K, n0, n1, fn):
    if n0 % 8 and fn != "e2_i8_gemm_scalar":
        # the SIMD kernels load whole 8-row groups from n0 and need it 8-aligned (every hot caller's
        # claims are; src/int8.c:157-161); only the scalar kernel takes an arbitrary column range
        n0 = 8
    rng = np.random.default_rng(M * N + K)
    lib = of.ref(blk)
    x = syn.activations(rng, M, K)
    w = of.Weight((rng.standard_normal((N, K)) * 0.05).astype(np.float32), blk, lib)
    qa, sa = of.quantize_biased(x, blk, lib=lib, fn="e2_quantize_blocks_avx512")
    ry = np.full((M, N), -777.0, np.float32)
    getattr(lib, fn)(ry.ctypes.data_as(of.f32p), qa.view(np.int8).ctypes.data_as(of.i8p), sa.ctypes.data_as(of.f32p),
                     C.byref(w.q), M, N, n0, n1)
    py = np.full((M, N), -777.0, np.float32)
    of.port().e2o_i8_gemm(py.ctypes.data_as(of.f32p), qa.view(np.int8).ctypes.data_as(of.i8p),
                          sa.ctypes.data_as(of.f32p), C.byref(w.q), M, N, n0, n1, blk)
    if fn == "e2_i8_gemm_avx2" or (fn == "e2_i8_gemm_scalar" and K > blk):
        # the AVX2 and scalar kernels fold blocks with a rounded multiply then an add
        # (src/kernels_i8_avx2.c, src/int8.c:144-145) where the AVX-512 kernel issues an FMA: the
        # int32 dots are the same, a multi-block fp32 sum differs in the last bits
        np.testing.assert_allclose(py, ry, rtol=1e-5, atol=1e-6)
    else:
        assert np.array_equal(py.view(np.int32), ry.view(np.int32))
    # the signed-operand form the device uses gives the same bits (no +128 zero point)
    if fn == "e2_i8_gemm_avx512":
        ys = of.gemm_plain((qa.astype(np.int16) - 128).astype(np.int8), sa, w.plain(), w.scales(), blk)
        assert np.array_equal(ys[:, n0:n1].view(np.int32), ry[:, n0:n1].view(np.int32))


def test_gemm_clamped_output(of, syn):
    rng = np.random.default_rng(8)
    lib = of.ref(128)
    x = syn.activations(rng, 8, 256)
    w = of.Weight((rng.standard_normal((64, 256)) * 0.1).astype(np.float32), 128, lib)
    w.q.out_min, w.q.out_max = -0.5, 0.5
    qa, sa = of.quantize_biased(x, 128, lib=lib, fn="e2_quantize_blocks_avx512")
    ry, py = np.empty((8, 64), np.float32), np.empty((8, 64), np.float32)
    lib.e2_i8_gemm_avx512(ry.ctypes.data_as(of.f32p), qa.view(np.int8).ctypes.data_as(of.i8p), sa.ctypes.data_as(of.f32p),
                          C.byref(w.q), 8, 64, 0, 64)
    of.port().e2o_i8_gemm(py.ctypes.data_as(of.f32p), qa.view(np.int8).ctypes.data_as(of.i8p), sa.ctypes.data_as(of.f32p),
                          C.byref(w.q), 8, 64, 0, 64, 128)
    assert np.array_equal(ry, py) and ry.max() <= 0.5 and ry.min() >= -0.5


def test_fp32_vtable_close_to_reference(of, syn):
    """RMSNorm / softmax / GELU-tanh agree to a few ulp. The reference is built -ffast-math:
    GCC turns GELU's 2/(e+1) into rcp14 + one Newton step and reassociates the final
    products, and sums norms in 16 lanes, so bit-exactness is not defined for these."""
    rng = np.random.default_rng(12)
    k = C.cast(of.mux().e2refmux_kernels(128), C.POINTER(C.c_void_p))
    # e2o_kernels layout: name, ablk(int, padded), then function pointers in declaration order
    fields = ["quantize", "gemm", "q8w_from_f32", "q8w_free", "rmsnorm", "norm_split", "norm_add", "gelu_tanh", "mul",
              "softmax"]
    ptr = {f: k[2 + i] for i, f in enumerate(fields)}
    gelu = C.CFUNCTYPE(None, of.f32p, C.c_size_t)(ptr["gelu_tanh"])
    x = (rng.standard_normal(4096) * 3).astype(np.float32)
    a, b = x.copy(), x.copy()
    gelu(a.ctypes.data_as(of.f32p), a.size)
    of.port().e2o_gelu_tanh(b.ctypes.data_as(of.f32p), b.size)
    np.testing.assert_allclose(b, a, rtol=2e-6, atol=1e-7)
    rms = C.CFUNCTYPE(None, of.f32p, C.c_int, C.c_int, of.f32p, C.c_float)(ptr["rmsnorm"])
    X = (rng.standard_normal((32, 768)) * 2).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(768)).astype(np.float32)
    r, p = X.copy(), X.copy()
    rms(r.ctypes.data_as(of.f32p), 32, 768, g.ctypes.data_as(of.f32p), 1e-6)
    of.port().e2o_rmsnorm(p.ctypes.data_as(of.f32p), 32, 768, g.ctypes.data_as(of.f32p), 1e-6)
    np.testing.assert_allclose(p, r, rtol=2e-6, atol=1e-7)
    sm = C.CFUNCTYPE(None, of.f32p, C.c_int)(ptr["softmax"])
    s = (rng.standard_normal(700) * 4).astype(np.float32)
    r, p = s.copy(), s.copy()
    sm(r.ctypes.data_as(of.f32p), 700)
    of.port().e2o_softmax(p.ctypes.data_as(of.f32p), 700)
    np.testing.assert_allclose(p, r, rtol=1e-5, atol=1e-9)


def test_ffn_block_port_vs_reference(of, syn):
    rng = np.random.default_rng(31)
    M, D, I = 64, 768, 1152
    x = rng.standard_normal((M, D)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    for ablk in (0, 128):
        # e2_q8w carries per-block weight sums, so a weight is packed for the activation block it meets
        r = np.random.default_rng(32)
        wg, wu = syn.packed_weight(r, I, D, 0.02, ablk or D), syn.packed_weight(r, I, D, 0.02, ablk or D)
        wd = syn.packed_weight(r, D, I, 0.02, ablk or I)
        yp, sp = of.ffn_block("port", x, g, 1e-6, wg, wu, wd, ablk=ablk, stages=True)
        yr, sr = of.ffn_block("reference", x, g, 1e-6, wg, wu, wd, ablk=ablk, stages=True)
        d = np.abs(sp["xq"].astype(int) - sr["xq"].astype(int))
        assert d.max() <= 1 and (d == 0).mean() > 0.999
        err = np.linalg.norm(yp - yr, axis=1) / np.linalg.norm(yr, axis=1)
        assert err.max() < 1e-4


def test_encoder_port_vs_reference(of, syn):
    cfg = syn.EncoderConfig(n_layers=2, hidden=256, n_heads=2, ffn=512, vocab=1000, dense_hidden=512, out_dim=256,
                            max_seq=64)
    w = syn.encoder_weights(cfg, seed=5)
    rng = np.random.default_rng(3)
    ids = syn.token_batch(rng, 3, 40, cfg.vocab)
    valid = np.ones((3, 40), np.uint8)
    valid[1, 30:] = 0
    valid[2] = 0
    p = of.encoder_forward("port", w, ids, valid)
    r = of.encoder_forward("reference", w, ids, valid)
    assert np.all(p[2] == 0) and np.all(r[2] == 0)
    assert cosine_rows(p[:2], r[:2]).min() >= 0.9999
