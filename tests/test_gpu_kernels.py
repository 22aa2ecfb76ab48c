"""Parity of the e2cuda kernels with the reference's CPU int8 path (through the C ABI, on a B200).

Bars: quantised bytes, scales, int32 dots and per-row-mode fp32 GEMM
outputs are bit-exact; fp32 epilogues that run after an RMSNorm are compared teacher-forced with
the reference's own tie rule; bf16 attention by cosine / relative error.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

from conftest import cosine_rows, tie_tolerant_bytes

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def f32_bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return np.array_equal(np.ascontiguousarray(a, np.float32).view(np.int32), np.ascontiguousarray(b, np.float32).view(np.int32))


# ------------------------------------------------------------------------------------------ A1 quantiser
QUANT_CASES = [(1, 768, 768), (7, 768, 768), (512, 768, 768), (333, 1152, 1152), (5, 8192, 8192), (17, 2048, 2048),
               (40000, 768, 768), (3001, 1152, 1152), (2500, 1024, 1024), (777, 128, 128),
               (9, 208, 208), (3, 3072, 3072), (64, 768, 128), (31, 1152, 128), (8, 512, 32), (8, 512, 64),
               (8, 1024, 256), (8, 1024, 512), (0, 768, 768)]


@pytest.mark.parametrize("M,K,ablk", QUANT_CASES)
def test_quantize_bitexact(e2c, of, syn, torch_cuda, M, K, ablk):
    rng = np.random.default_rng(M * 131 + K + ablk)
    x = syn.activations(rng, max(M, 1), K)[:M] * rng.uniform(1e-3, 10.0, (M, 1)).astype(np.float32)
    x = np.ascontiguousarray(x, np.float32)
    if M > 0:
        x[0] = 0.0                      # all-zero row: scale 1, bytes 0
    if M > 2:
        x[2, :ablk] = 0.0               # one all-zero block
    q, s = e2c.quantize_rows(dev(torch_cuda, x), ablk)
    eq, es = of.quantize_signed(x, ablk) if M else (np.zeros((0, K), np.int8), np.zeros((0, K // ablk), np.float32))
    assert np.array_equal(q.cpu().numpy(), eq)
    assert f32_bits_equal(s.cpu().numpy(), es)


def test_quantize_clamp_and_host_dropin(e2c, of, syn, torch_cuda):
    rng = np.random.default_rng(3)
    x = syn.activations(rng, 40, 512)
    lo, hi = -0.75, 0.5
    q, s = e2c.quantize_rows(dev(torch_cuda, x), 128, lo, hi)
    eb, es = of.quantize_biased(x, 128, lo, hi)
    assert np.array_equal(q.cpu().numpy().view(np.uint8) ^ 0x80, eb)
    assert f32_bits_equal(s.cpu().numpy(), es)
    # the reference-signature drop-in: host buffers, biased bytes, block from e2cuda_set_act_block
    lib = e2c.lib()
    lib.e2cuda_set_act_block(128)
    out = np.empty((40, 512), np.int8)
    sc = np.empty((40, 4), np.float32)
    lib.e2cuda_i8_quantize_host(out.ctypes.data_as(e2c.i8p), sc.ctypes.data_as(e2c.f32p), x.ctypes.data_as(e2c.f32p),
                                40, 512, -math.inf, math.inf)
    assert e2c.last_error() == ""
    eb2, es2 = of.quantize_biased(x, 128)
    assert np.array_equal(out.view(np.uint8), eb2) and f32_bits_equal(sc, es2)


# ------------------------------------------------------------------------------------------ A3 GEMM
GEMM_CASES = [
    (512, 1152, 768, 768),     # config 0
    (1, 256, 768, 768), (7, 40, 768, 768), (129, 300, 768, 768), (200, 1152, 1152, 1152),
    (64, 64, 2048, 2048), (33, 96, 208, 208), (300, 2304, 768, 768), (16, 512, 8192, 8192),
    (8, 64, 512, 128), (130, 256, 1024, 128), (17, 48, 384, 128), (256, 384, 2048, 256),
    # large enough for CTA pairs (256-row tiles over two SMs): 192-, 128- and 256-column tiles
    (2048, 2560, 256, 256), (4096, 1152, 768, 768), (9472, 512, 256, 256),
    # per-128-block scales on CTA pairs (M > 256, a wave of 256 x 128 pair tiles), incl. a ragged M
    (4096, 1152, 768, 128), (5000, 2048, 512, 128),
]


def _gemm_inputs(rng, M, N, K, ablk):
    nb = K // ablk
    qa = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    a_s = rng.uniform(1e-3, 0.05, size=(M, nb)).astype(np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.uniform(1e-4, 0.02, size=N).astype(np.float32)
    return qa, a_s, w, ws


@pytest.mark.parametrize("M,N,K,ablk", GEMM_CASES)
def test_gemm_bitexact(e2c, of, torch_cuda, M, N, K, ablk):
    rng = np.random.default_rng(M + 7 * N + K + ablk)
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, ablk)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = dev(torch_cuda, qa), dev(torch_cuda, a_s)
    y = e2c.i8_gemm(W, qd, sd, ablk).cpu().numpy()
    dots = e2c.i8_gemm(W, qd, sd, ablk, dots=True).cpu().numpy()
    e2c.check()
    ey, ed = of.gemm_plain(qa, a_s, w, ws, ablk, want_dots=True)
    assert np.array_equal(dots, ed), "int32 block dots differ"
    assert f32_bits_equal(y, ey), f"fp32 outputs differ: max abs {np.abs(y - ey).max()}"


@pytest.mark.parametrize("N,K,ablk", [(200, 768, 768), (77, 256, 128), (1152, 768, 768)])
def test_q8cache_upload_matches_the_repack(e2c, of, torch_cuda, tmp_path, N, K, ablk):
    """A11: a kind-4 cache entry (the device layout) goes to the GPU with one copy, a kind-3 entry
    through the repack; both compute bit-for-bit what e2cuda_w8_from_q8w's weight computes, and
    what the port computes."""
    rng = np.random.default_rng(N + K)
    w = of.Weight(rng.standard_normal((N, K)).astype(np.float32) * 0.05, ablk)
    wr = e2c.Q8CacheWriter(tmp_path / "c.e8cq")
    wr.put_w8("w4", w.q)
    wr.put_q8w("w3", w.q)
    wr.commit()
    c = e2c.Q8Cache(tmp_path / "c.e8cq")
    W4, W3 = c.upload_w8("w4"), c.upload_w8("w3")
    c.close()  # the device copies do not depend on the mapping
    Wr = e2c.Weight(q8w=C.cast(C.byref(w.q), C.POINTER(e2c.Q8W)).contents)
    assert (W4.w8.N, W4.w8.K, W4.w8.rows, W4.w8.ld) == (Wr.w8.N, Wr.w8.K, Wr.w8.rows, Wr.w8.ld)
    M = 300
    qa = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    a_s = rng.uniform(1e-3, 0.05, size=(M, K // ablk)).astype(np.float32)
    qd, sd = dev(torch_cuda, qa), dev(torch_cuda, a_s)
    ys = [e2c.i8_gemm(W, qd, sd, ablk).cpu().numpy() for W in (W4, W3, Wr)]
    e2c.check()
    ey = of.gemm_plain(qa, a_s, w.plain(), w.scales(), ablk)
    for y in ys:
        assert f32_bits_equal(y, ey)


def test_gemm_column_range_residual(e2c, of, torch_cuda):
    rng = np.random.default_rng(11)
    M, N, K = 45, 40, 768
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
    W = e2c.Weight(w=w, scale=ws)
    y0 = np.full((M, N), -777.0, np.float32)
    y = dev(torch_cuda, y0)
    res = rng.standard_normal((M, N)).astype(np.float32)
    e2c.i8_gemm(W, dev(torch_cuda, qa), dev(torch_cuda, a_s), K, n0=3, n1=29, residual=dev(torch_cuda, res), y=y)
    got = y.cpu().numpy()
    ey = of.gemm_plain(qa, a_s, w, ws, K)
    assert np.all(got[:, :3] == -777.0) and np.all(got[:, 29:] == -777.0), "columns outside [n0, n1) were written"
    assert f32_bits_equal(got[:, 3:29], ey[:, 3:29] + res[:, 3:29])


def test_gemm_residual_cta_pairs(e2c, of, torch_cuda):
    """The residual epilogue on 256-row tiles shared by a CTA pair, TMA-stored."""
    rng = np.random.default_rng(12)
    M, N, K = 9472, 512, 256
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
    W = e2c.Weight(w=w, scale=ws)
    res = rng.standard_normal((M, N)).astype(np.float32)
    y = e2c.i8_gemm(W, dev(torch_cuda, qa), dev(torch_cuda, a_s), K, residual=dev(torch_cuda, res)).cpu().numpy()
    e2c.check()
    assert f32_bits_equal(y, of.gemm_plain(qa, a_s, w, ws, K) + res)


def test_gemm_host_dropin_matches_reference_kernel(e2c, of, syn, torch_cuda):
    """e2cuda_i8_gemm_host has e2_i8_gemm_fn's signature: biased bytes, packed e2_q8w, row stride N,
    columns [n0, n1). Both modes, against the port of src/kernels_i8_avx512_vnni.c."""
    rng = np.random.default_rng(5)
    for ablk, M, N, K in ((768, 37, 200, 768), (128, 20, 96, 512)):
        x = syn.activations(rng, M, K)
        pw = syn.packed_weight(rng, N, K, 0.02, ablk)
        qb, qs = of.quantize_biased(x, ablk)
        q8 = of.Q8W()
        pw.fill(q8)
        want = np.full((M, N), -5.0, np.float32)
        of.port().e2o_i8_gemm(want.ctypes.data_as(of.f32p), qb.view(np.int8).ctypes.data_as(of.i8p),
                              qs.ctypes.data_as(of.f32p), C.byref(q8), M, N, 8, N - 5, ablk)
        got = np.full((M, N), -5.0, np.float32)
        q8e = e2c.Q8W()
        pw.fill(q8e)
        e2c.lib().e2cuda_i8_gemm_host(got.ctypes.data_as(e2c.f32p), qb.view(np.int8).ctypes.data_as(e2c.i8p),
                                      qs.ctypes.data_as(e2c.f32p), C.byref(q8e), M, N, 8, N - 5)
        assert e2c.last_error() == "", e2c.last_error()
        assert f32_bits_equal(got, want)
    e2c.lib().e2cuda_host_cache_clear()


def test_gemm_host_dropin_from_concurrent_pool_workers(e2c, of, syn, torch_cuda):
    """e2.c calls e2_i8_gemm from every pool worker at once, each on its own column range
    (src/text.c:301-318): four threads calling the drop-in together give the single-call bits."""
    import threading

    rng = np.random.default_rng(15)
    M, N, K, ablk = 48, 512, 768, 768
    x = syn.activations(rng, M, K)
    pw = syn.packed_weight(rng, N, K, 0.02, ablk)
    qb, qs = of.quantize_biased(x, ablk)
    q8 = of.Q8W()
    pw.fill(q8)
    want = np.empty((M, N), np.float32)
    of.port().e2o_i8_gemm(want.ctypes.data_as(of.f32p), qb.view(np.int8).ctypes.data_as(of.i8p),
                          qs.ctypes.data_as(of.f32p), C.byref(q8), M, N, 0, N, ablk)
    q8e = e2c.Q8W()
    pw.fill(q8e)
    got = np.full((M, N), -5.0, np.float32)
    errors = []

    def worker(n0, n1):
        for _ in range(5):
            e2c.lib().e2cuda_i8_gemm_host(got.ctypes.data_as(e2c.f32p), qb.view(np.int8).ctypes.data_as(e2c.i8p),
                                          qs.ctypes.data_as(e2c.f32p), C.byref(q8e), M, N, n0, n1)
            if e2c.last_error():
                errors.append(e2c.last_error())

    threads = [threading.Thread(target=worker, args=(128 * t, 128 * t + 128)) for t in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    e2c.lib().e2cuda_host_cache_clear()
    assert not errors, errors
    assert f32_bits_equal(got, want)


def test_gemm_clamp_from_q8w(e2c, of, syn, torch_cuda):
    rng = np.random.default_rng(9)
    M, N, K = 30, 64, 256
    pw = syn.packed_weight(rng, N, K, 0.05, K)
    q8 = e2c.Q8W()
    pw.fill(q8)
    q8.out_min, q8.out_max = -0.5, 0.5  # the audio tower's clipped linears (e2.c src/int8.h:84-88)
    W = e2c.Weight(q8w=q8)
    x = syn.activations(rng, M, K)
    qa, a_s = of.quantize_signed(x, K)
    y = e2c.i8_gemm(W, dev(torch_cuda, qa), dev(torch_cuda, a_s), K).cpu().numpy()
    ey = of.gemm_plain(qa, a_s, pw.q, pw.scale, K, out_min=-0.5, out_max=0.5)
    assert f32_bits_equal(y, ey) and y.max() <= 0.5 and y.min() >= -0.5


# ------------------------------------------------------------------------------------------ fused epilogues
def _launch(e2c, args, torch):
    lib = e2c.lib()
    lib.e2c_msg.restype = C.c_char_p
    rc = lib.e2c_gemm(C.byref(args), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.e2c_msg().decode()
    e2c.check()


def _args_for(W, qd, sd, M, K):
    from conftest import load_e2c

    a = load_e2c().GemmArgs()
    a.a, a.lda, a.a_scale = qd.data_ptr(), W.w8.ld, sd.data_ptr()
    a.w, a.ldw, a.wrows, a.w_scale = C.cast(W.w8.w, C.c_void_p), W.w8.ld, W.w8.rows, C.cast(W.w8.scale, C.c_void_p)
    a.M, a.K, a.ablk, a.n0, a.n1 = M, K, K, 0, W.N
    a.out_min, a.out_max = -1e31, 1e31
    return a


@pytest.mark.parametrize("M", [150, 2176])  # 2176 rows: enough 256-row tiles for CTA pairs
def test_gelu_gate_epilogue(e2c, of, torch_cuda, M):
    """gate|up GEMM with GELU-tanh(g)*u in the epilogue (e2.c src/text.c:424-447 +
    src/kernels_avx512.c:186-203). g and u are the bit-exact dequantised GEMM outputs; GELU is a
    floating-point epilogue (the reference's -ffast-math build is itself not reproducible to the
    bit), so h agrees with the port within 2e-6 relative (a few ulp)."""
    torch = torch_cuda
    rng = np.random.default_rng(21 + M)
    D, I = 768, 1152
    qa, a_s, wg, sg = _gemm_inputs(rng, M, I, D, D)
    _, _, wu, su = _gemm_inputs(rng, M, I, D, D)
    wi = np.empty((2 * I, D), np.int8)
    si = np.empty(2 * I, np.float32)
    for t in range(I // 128):
        wi[256 * t:256 * t + 128], si[256 * t:256 * t + 128] = wg[128 * t:128 * t + 128], sg[128 * t:128 * t + 128]
        wi[256 * t + 128:256 * t + 256], si[256 * t + 128:256 * t + 256] = wu[128 * t:128 * t + 128], su[128 * t:128 * t + 128]
    W = e2c.Weight(w=wi, scale=si)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    h = torch.zeros((M, I), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, D)
    a.epi, a.y, a.ldy = 3, h.data_ptr(), I
    _launch(e2c, a, torch)
    g = of.gemm_plain(qa, a_s, wg, sg, D)
    u = of.gemm_plain(qa, a_s, wu, su, D)
    gg = np.ascontiguousarray(g.copy())
    of.port().e2o_gelu_tanh(gg.ctypes.data_as(of.f32p), gg.size)
    want = (gg * u).astype(np.float32)
    got = h.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7 * float(np.abs(want).max()))
    # and the bytes a per-token requantisation of h makes agree within the reference's tie rule
    gq, gs = of.quantize_signed(np.ascontiguousarray(got), I)
    wq, ws = of.quantize_signed(np.ascontiguousarray(want), I)
    tie_tolerant_bytes(gq, wq, want * (np.float32(127.0) / np.abs(want).max(axis=1, keepdims=True)))


def _gate_up_weight(e2c, rng, M, D, I):
    """Inputs and the interleaved gate|up weight (groups of 128 gate rows, then 128 up rows)."""
    qa, a_s, wg, sg = _gemm_inputs(rng, M, I, D, D)
    _, _, wu, su = _gemm_inputs(rng, M, I, D, D)
    wi = np.empty((2 * I, D), np.int8)
    si = np.empty(2 * I, np.float32)
    for t in range(I // 128):
        wi[256 * t:256 * t + 128], si[256 * t:256 * t + 128] = wg[128 * t:128 * t + 128], sg[128 * t:128 * t + 128]
        wi[256 * t + 128:256 * t + 256], si[256 * t + 128:256 * t + 256] = wu[128 * t:128 * t + 128], su[128 * t:128 * t + 128]
    return qa, a_s, e2c.Weight(w=wi, scale=si)


@pytest.mark.parametrize("M,I", [(300, 1152), (16384, 1152), (1000, 128), (517, 2048), (129, 1024)])
def test_gelu_quant_epilogue(e2c, of, torch_cuda, M, I):
    """gate|up GEMM with GELU-gate and the per-token quantiser of h in the epilogue (h never stored):
    the int8 rows and scales are bit-identical to the GELU epilogue followed by the quantiser kernel
    (both already checked against the reference above). Rows span a cluster of I / 128 CTAs (1 to 16,
    9 for the encoder's I = 1152); 16384 rows give every CTA several row blocks."""
    torch = torch_cuda
    rng = np.random.default_rng(91 + M + I)
    D = 768
    qa, a_s, W = _gate_up_weight(e2c, rng, M, D, I)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    lib = e2c.lib()
    if not lib.e2c_gemm_gelu_quant_supported(I // 128):
        pytest.skip(f"the device holds no cluster of {I // 128} CTAs")
    h = torch.zeros((M, I), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, D)
    a.epi, a.y, a.ldy = e2c.EPI_GELU, h.data_ptr(), I
    _launch(e2c, a, torch)
    want_q, want_s = e2c.quantize_rows(h, I)
    q = torch.full((M, I), 99, dtype=torch.int8, device="cuda")
    s = torch.zeros((M,), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, D)
    a.epi, a.q8, a.ldq, a.q8_scale = e2c.EPI_GELUQ, q.data_ptr(), I, s.data_ptr()
    _launch(e2c, a, torch)
    assert np.array_equal(q.cpu().numpy(), want_q.cpu().numpy())
    assert f32_bits_equal(s.cpu().numpy(), want_s.cpu().numpy()[:, 0])


@pytest.mark.parametrize("B,S", [(2, 200), (16, 240)])  # 16 x 240 rows: CTA pairs
def test_qkv_epilogue_norm_rope(e2c, of, torch_cuda, B, S):
    """q|k|v GEMM with per-head RMSNorm (+gamma) and RoPE in the epilogue (e2.c src/text.c:836-854),
    bf16 outputs, V transposed. fp32 differs from the port only by the sum order of the norm."""
    torch = torch_cuda
    rng = np.random.default_rng(31)
    D, H, Dh = 768, 3, 256
    M, N = B * S, (H + 2) * Dh
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, D, D)
    qg = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    kg = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    cs = np.empty((S, Dh), np.float32)
    sn = np.empty((S, Dh), np.float32)
    of.port().e2o_rope_tables(cs.ctypes.data_as(of.f32p), sn.ctypes.data_as(of.f32p), S, Dh, 10000.0)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    ldvt = (S + 7) // 8 * 8
    Q = torch.zeros((M, H * Dh), dtype=torch.bfloat16, device="cuda")
    K = torch.zeros((M, Dh), dtype=torch.bfloat16, device="cuda")
    Vt = torch.zeros((B, Dh, ldvt), dtype=torch.bfloat16, device="cuda")
    gq, gk = dev(torch, qg), dev(torch, kg)
    # the kernel's tables are pair-major: [128][ldrope], ldrope >= S (padded here to check the stride)
    ldrope = S + 5
    cT = np.zeros((128, ldrope), np.float32)
    sT = np.zeros((128, ldrope), np.float32)
    cT[:, :S], sT[:, :S] = cs[:, :128].T, sn[:, :128].T
    cd, sdn = dev(torch, cT), dev(torch, sT)
    a = _args_for(W, qd, sd, M, D)
    a.epi, a.nq = 4, H
    a.q_out, a.k_out, a.vt_out, a.ldvt, a.seq_len = Q.data_ptr(), K.data_ptr(), Vt.data_ptr(), ldvt, S
    a.q_gamma, a.k_gamma, a.rope_cos, a.rope_sin, a.eps = gq.data_ptr(), gk.data_ptr(), cd.data_ptr(), sdn.data_ptr(), 1e-6
    a.ldrope = ldrope
    _launch(e2c, a, torch)
    y = of.gemm_plain(qa, a_s, w, ws, D).reshape(M, H + 2, Dh)
    port = of.port()
    exp = np.empty_like(y)
    for hd in range(H + 2):
        blk = np.ascontiguousarray(y[:, hd])
        gamma = qg if hd < H else (kg if hd == H else None)
        port.e2o_rmsnorm(blk.ctypes.data_as(of.f32p), M, Dh, None if gamma is None else gamma.ctypes.data_as(of.f32p), 1e-6)
        if hd <= H:
            port.e2o_rope_rows(blk.ctypes.data_as(of.f32p), 0, M, 1, Dh, Dh,
                               np.ascontiguousarray(np.tile(cs, (B, 1))).ctypes.data_as(of.f32p),
                               np.ascontiguousarray(np.tile(sn, (B, 1))).ctypes.data_as(of.f32p))
        exp[:, hd] = blk
    to_bf = lambda t: t.float().cpu().numpy()
    got = np.concatenate([to_bf(Q).reshape(M, H, Dh), to_bf(K).reshape(M, 1, Dh),
                          to_bf(Vt)[:, :, :S].transpose(0, 2, 1).reshape(M, 1, Dh)], axis=1)
    want = torch.from_numpy(exp).to(torch.bfloat16).float().numpy()
    diff = np.abs(got - want)
    # One bf16 ulp, plus an absolute floor for RoPE's cancellations: a*cos - b*sin near zero keeps
    # the fp32 rounding differences of its O(1) normalised inputs (~1e-7), which can exceed an ulp
    # of the tiny result. The floor is 30 fp32 ulps at 1.0, far below any real error.
    tol = np.abs(want) * 2.0 ** -7 + 4e-6
    assert np.all(diff <= tol), f"beyond one bf16 ulp: {int((diff > tol).sum())}, worst {diff.max()}"
    assert (diff == 0).mean() > 0.99


@pytest.mark.parametrize("M,D,final", [(300, 768, False), (16384, 768, False), (1000, 768, True), (700, 256, False),
                                       (517, 1024, False), (130, 128, False), (4000, 1024, True)])
def test_gemm_norm_add_epilogue(e2c, of, torch_cuda, M, D, final):
    """o_proj / down with the residual norm fused (e2.c src/text.c:947,950 + :321-339): the GEMM's fp32
    output t stays on chip; x = rmsnorm(t) * g1 + res becomes the residual and the next layer's input
    rmsnorm(x) * g2 is quantised per token (or, after the last layer, rmsnorm(x) * gf is written).
    Rows span a cluster of D / 128 CTAs (1 to 8). Against fp64 of the same formula on the bit-exact
    t; 16384 rows give every CTA several row blocks, so the pipelined epilogue wraps its slots."""
    torch = torch_cuda
    rng = np.random.default_rng(61 + M)
    N = K = D
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
    res0 = rng.standard_normal((M, N)).astype(np.float32)
    g1 = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    g2 = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    eps = 1e-6
    W = e2c.Weight(w=w, scale=ws)
    res = dev(torch, res0)
    q = torch.zeros((M, N), dtype=torch.int8, device="cuda")
    qs = torch.zeros((M,), dtype=torch.float32, device="cuda")
    gd1, gd2 = dev(torch, g1), dev(torch, g2)
    a = _args_for(W, dev(torch, qa), dev(torch, a_s), M, K)
    a.epi, a.eps = e2c.EPI_NORMADD, eps
    a.res, a.ldres, a.norm_g1 = res.data_ptr(), N, gd1.data_ptr()
    if final:
        a.norm_gf = gd2.data_ptr()
    else:
        a.norm_g2, a.q8, a.ldq, a.q8_scale = gd2.data_ptr(), q.data_ptr(), N, qs.data_ptr()
    _launch(e2c, a, torch)
    t = of.gemm_plain(qa, a_s, w, ws, K).astype(np.float64)
    inv1 = 1.0 / np.sqrt((t * t).mean(axis=1, keepdims=True) + eps)
    x = t * inv1 * g1 + res0
    inv2 = 1.0 / np.sqrt((x * x).mean(axis=1, keepdims=True) + eps)
    z = x * inv2 * g2
    got = res.cpu().numpy()
    want = z if final else x
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    assert err.max() < 1e-5, f"residual off by {err.max()}"
    if not final:
        amax = np.abs(z).max(axis=1, keepdims=True)
        np.testing.assert_allclose(qs.cpu().numpy(), amax[:, 0] / 127.0, rtol=1e-5)
        pre = z * (127.0 / amax)
        tie_tolerant_bytes(q.cpu().numpy(), np.clip(np.rint(pre), -127, 127).astype(np.int8), pre)


@pytest.mark.parametrize("M,D,K,mode", [(300, 768, 768, "g2"), (4096, 768, 1152, "g2"), (1000, 768, 768, "final"),
                                        (517, 1024, 1024, "g2"), (700, 512, 2048, "x"), (130, 128, 256, "g2"),
                                        (16384, 512, 512, "ls"), (1000, 512, 1024, "x")])
def test_gemm_norm_add_epilogue_per_block(e2c, of, torch_cuda, M, D, K, mode):
    """The residual norms fused into o_proj / down with per-128-block activation scales (e2.c's
    default recipe): t is the per-block fold (bit-exact to the port's GEMM), x = rmsnorm(t) * g1 + res
    (times the layer scalar in mode "ls", as e2.c's text tower's per-layer-embedding step) becomes the
    residual, and rmsnorm(x) * g2 is quantised per 128-column block (scales [M][D/128]); mode "x"
    quantises x itself (the text tower after its FFN), "final" writes rmsnorm(x) * gf. Against fp64
    of the same formula on the bit-exact t; bytes within the tie rule. D = 1024 takes the three-stage
    kernel, 16384 rows wrap the pipelined epilogue's slots many times."""
    final = mode == "final"
    ls = 0.6875 if mode == "ls" else 1.0
    torch = torch_cuda
    rng = np.random.default_rng(67 + M + K)
    N = D
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, 128)
    res0 = rng.standard_normal((M, N)).astype(np.float32)
    g1 = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    g2 = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    eps = 1e-6
    W = e2c.Weight(w=w, scale=ws)
    res = dev(torch, res0)
    q = torch.zeros((M, N), dtype=torch.int8, device="cuda")
    qs = torch.zeros((M, N // 128), dtype=torch.float32, device="cuda")
    gd1, gd2 = dev(torch, g1), dev(torch, g2)
    a = _args_for(W, dev(torch, qa), dev(torch, a_s), M, K)
    a.ablk, a.epi, a.eps, a.norm_ls = 128, e2c.EPI_NORMADD, eps, ls
    a.res, a.ldres, a.norm_g1 = res.data_ptr(), N, gd1.data_ptr()
    if final:
        a.norm_gf = gd2.data_ptr()
    else:
        a.q8, a.ldq, a.q8_scale = q.data_ptr(), N, qs.data_ptr()
        if mode != "x":
            a.norm_g2 = gd2.data_ptr()
    _launch(e2c, a, torch)
    t = of.gemm_plain(qa, a_s, w, ws, 128).astype(np.float64)
    inv1 = 1.0 / np.sqrt((t * t).mean(axis=1, keepdims=True) + eps)
    x = (t * inv1 * g1 + res0) * ls
    inv2 = 1.0 / np.sqrt((x * x).mean(axis=1, keepdims=True) + eps)
    z = x if mode == "x" else x * inv2 * g2
    got = res.cpu().numpy()
    want = z if final else x
    err = np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)
    assert err.max() < 1e-5, f"residual off by {err.max()}"
    if not final:
        zb = z.reshape(M, N // 128, 128)
        amax = np.abs(zb).max(axis=2, keepdims=True)
        np.testing.assert_allclose(qs.cpu().numpy(), amax[:, :, 0] / 127.0, rtol=1e-5)
        pre = (zb * (127.0 / amax)).reshape(M, N)
        tie_tolerant_bytes(q.cpu().numpy(), np.clip(np.rint(pre), -127, 127).astype(np.int8), pre)


def test_norm_quant_teacher_forced(e2c, of, torch_cuda):
    """The config-1 prologue (rmsnorm * gamma -> per-row quantise): bytes within the tie rule."""
    torch = torch_cuda
    rng = np.random.default_rng(41)
    M, D = 300, 768
    x = rng.standard_normal((M, D)).astype(np.float32) * 3
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    q = torch.zeros((M, D), dtype=torch.int8, device="cuda")
    s = torch.zeros((M, 1), dtype=torch.float32, device="cuda")
    lib = e2c.lib()
    lib.e2c_norm_quant.argtypes = [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    xd, gd = dev(torch, x), dev(torch, g)
    assert lib.e2c_norm_quant(xd.data_ptr(), gd.data_ptr(), 1e-6, q.data_ptr(), s.data_ptr(), M, D, D,
                              torch.cuda.current_stream().cuda_stream) == 0
    e2c.check()
    xn = x.copy()
    of.port().e2o_rmsnorm(xn.ctypes.data_as(of.f32p), M, D, g.ctypes.data_as(of.f32p), 1e-6)
    eq, es = of.quantize_signed(xn, D)
    np.testing.assert_allclose(s.cpu().numpy(), es, rtol=2e-6)  # normed values differ by a few ulp (sum order)
    pre = xn * (np.float32(127.0) / np.abs(xn).max(axis=1, keepdims=True))
    tie_tolerant_bytes(q.cpu().numpy(), eq, pre)


# ------------------------------------------------------------------------------------------ A8 attention
def _attn_ref(q, k, v, valid, B, S, H, scale):
    """fp64 attention over the valid keys of each sequence; invalid query rows are 0."""
    Dh = 256
    out = np.zeros((B * S, H * Dh), np.float64)
    for b in range(B):
        keys = np.arange(S) if valid is None else np.nonzero(valid[b])[0]
        kb = k[b * S + keys].astype(np.float64)
        vb = v[b * S + keys].astype(np.float64)
        for h in range(H):
            qh = q[b * S:(b + 1) * S, h * Dh:(h + 1) * Dh].astype(np.float64)
            if len(keys) == 0:
                continue
            lg = qh @ kb.T * scale
            lg -= lg.max(axis=1, keepdims=True)
            p = np.exp(lg)
            p /= p.sum(axis=1, keepdims=True)
            o = p @ vb
            if valid is not None:
                o[valid[b] == 0] = 0
            out[b * S:(b + 1) * S, h * Dh:(h + 1) * Dh] = o
    return out


@pytest.mark.parametrize("B,S,H,scale,masked", [(2, 300, 3, 1 / 16, True), (3, 512, 3, 1 / 16, False),
                                                (1, 64, 3, 1 / 16, False), (2, 1, 3, 1 / 16, False),
                                                (2, 700, 3, 1.0, True), (1, 130, 1, 1 / 16, False),
                                                # more units (sequence, head, query tile) than SMs: the
                                                # persistent CTAs carry state from one unit to the next
                                                (16, 512, 3, 1 / 16, False), (24, 300, 3, 1 / 16, True),
                                                (150, 64, 1, 1 / 16, True)])
def test_attention_vs_fp64(e2c, torch_cuda, B, S, H, scale, masked):
    torch = torch_cuda
    rng = np.random.default_rng(S * 10 + B)
    Dh = 256
    qf = torch.from_numpy(rng.standard_normal((B * S, H * Dh)).astype(np.float32)).to(torch.bfloat16)
    kf = torch.from_numpy(rng.standard_normal((B * S, Dh)).astype(np.float32)).to(torch.bfloat16)
    vf = torch.from_numpy(rng.standard_normal((B * S, Dh)).astype(np.float32)).to(torch.bfloat16)
    valid = None
    if masked:
        valid = np.ones((B, S), np.uint8)
        valid[-1, S - S // 6:] = 0
        valid[0, 5:9] = 0
    ldvt = (S + 7) // 8 * 8
    vt = torch.zeros((B, Dh, ldvt), dtype=torch.bfloat16)
    vt[:, :, :S] = vf.reshape(B, S, Dh).transpose(1, 2)
    vd = None if valid is None else dev(torch, valid.reshape(-1))
    ctx = e2c.attention(qf.cuda(), kf.cuda(), vt.cuda(), vd, B, S, H, scale)
    e2c.check()
    got = ctx.cpu().numpy()
    want = _attn_ref(qf.float().numpy(), kf.float().numpy(), vf.float().numpy(), valid, B, S, H, scale)
    for b in range(B):
        for h in range(H):
            rows = slice(b * S, (b + 1) * S)
            g = got[rows, h * Dh:(h + 1) * Dh]
            w = want[rows, h * Dh:(h + 1) * Dh]
            live = np.linalg.norm(w, axis=1) > 0
            if valid is not None:
                assert np.all(g[valid[b] == 0] == 0)
            err = np.linalg.norm(g[live] - w[live], axis=1) / np.linalg.norm(w[live], axis=1)
            assert err.max() < 1e-2, f"b={b} h={h} worst row rel err {err.max()}"
            assert cosine_rows(g[live], w[live]).min() > 0.9999


# ------------------------------------------------------------------------------------------ failure detection
def test_bounded_wait_expires_and_reports(e2c, torch_cuda):
    """The bounded mbarrier wait every kernel uses (ptx.cuh mbar_wait): with its arrival withheld it
    gives up after its ~2 s bound, records the code in the device status word and returns, so
    e2cuda_check reports the failure and the context keeps working. With the arrival it completes
    at once and records nothing."""
    import time

    torch = torch_cuda
    lib = e2c.lib()
    lib.e2c_wait_selftest.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.e2c_wait_selftest.restype = C.c_int
    lib.e2cu_status.restype = C.c_void_p
    e2c.check()  # start from a clean status word
    status = lib.e2cu_status()
    done = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.e2c_wait_selftest(status, 0x102, 1, done.data_ptr(), stream) == 0
    e2c.check()
    assert int(done.item()) == 1
    t0 = time.perf_counter()
    assert lib.e2c_wait_selftest(status, 0x102, 0, done.data_ptr(), stream) == 0
    with pytest.raises(e2c.E2CudaError, match="0x102"):
        e2c.check()
    waited = time.perf_counter() - t0
    assert int(done.item()) == 0
    assert 1.5 < waited < 30, waited
    # the status was cleared by the check and the device still runs kernels
    x = torch.randn((64, 768), device="cuda")
    q, s = e2c.quantize_rows(x, 768)
    e2c.check()
    assert q.shape == (64, 768)


# ------------------------------------------------------------------------------------------ short-M GEMM
STREAM_CASES = [
    # (M, N, K): the config-3 weights at M = 1 and 16, token counts around each MMA width, ragged
    # N and K (partial weight tiles, zero-filled k-blocks), tiny problems (fewer tiles than SMs)
    (1, 8192, 2048), (16, 8192, 2048), (1, 2048, 8192), (16, 2048, 8192), (1, 2048, 2048), (16, 2048, 2048),
    (2, 1152, 768), (7, 768, 1152), (17, 1152, 768), (33, 768, 768), (64, 3072, 768), (100, 768, 3072),
    (128, 8192, 2048), (200, 2048, 2048), (256, 1152, 768), (5, 300, 208), (16, 16, 128), (3, 130, 4096),
]


def _stream_gemm(e2c, torch, W, qd, sd, M, resid=None, n0=0, n1=None):
    """The weight-streaming kernel itself (e2c_gemm_stream) with a zeroed workspace."""
    lib = e2c.lib()
    lib.e2c_gemm_stream.argtypes = [C.POINTER(e2c.GemmArgs), C.c_void_p]
    lib.e2c_gemm_stream.restype = C.c_int
    lib.e2c_gemm_ws_bytes.argtypes = [C.c_int]
    lib.e2c_gemm_ws_bytes.restype = C.c_size_t
    lib.e2cu_status.restype = C.c_void_p
    n1 = W.N if n1 is None else n1
    wsb = lib.e2c_gemm_ws_bytes(M)
    ws = torch.zeros(wsb // 4 + 32, dtype=torch.int32, device="cuda")
    y = torch.full((M, W.N), float("nan"), dtype=torch.float32, device="cuda")
    a = e2c.gemm_args(W, qd, sd, M)
    a.n0, a.n1 = n0, n1
    a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), W.N
    if resid is not None:
        a.epi, a.resid, a.ldr = e2c.EPI_RESID, resid.data_ptr(), W.N
    a.ws, a.ws_bytes = ws.data_ptr(), wsb
    a.status = lib.e2cu_status()
    assert lib.e2c_gemm_stream(C.byref(a), torch.cuda.current_stream().cuda_stream) == 0, lib.e2c_msg().decode()
    e2c.check()
    return y, ws


@pytest.mark.parametrize("M,N,K", STREAM_CASES)
def test_stream_gemm_bitexact(e2c, of, torch_cuda, M, N, K):
    """The weight-streaming kernel (weight rows in the MMA's M slot, stream-K over the SMs, split
    tiles reduced through the workspace) against the reference fold, bit for bit; the workspace is
    zero again afterwards; the op API's GEMM (per-stream workspace) gives the same bits."""
    torch = torch_cuda
    rng = np.random.default_rng(M * 7 + N + 3 * K)
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    y, wsp = _stream_gemm(e2c, torch, W, qd, sd, M)
    ey = of.gemm_plain(qa, a_s, w, ws, K)
    assert f32_bits_equal(y.cpu().numpy(), ey), f"max abs diff {np.abs(y.cpu().numpy() - ey).max()}"
    assert int(wsp.abs().sum().item()) == 0, "workspace not returned to zero"
    y2 = e2c.i8_gemm(W, qd, sd, K).cpu().numpy()
    e2c.check()
    assert f32_bits_equal(y2, ey)


def test_stream_gemm_residual_clamp_and_columns(e2c, of, torch_cuda):
    """Residual epilogue, the e2_q8w output clamp and a column range [n0, n1) on the streaming
    kernel; columns outside the range stay untouched."""
    torch = torch_cuda
    rng = np.random.default_rng(77)
    M, N, K = 12, 1000, 1536
    qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
    W = e2c.Weight(w=w, scale=ws)
    W.w8.out_min, W.w8.out_max = -0.5, 0.75
    res = rng.standard_normal((M, N)).astype(np.float32)
    qd, sd, rd = dev(torch, qa), dev(torch, a_s), dev(torch, res)
    y, wsp = _stream_gemm(e2c, torch, W, qd, sd, M, resid=rd, n0=136, n1=900)
    ey = of.gemm_plain(qa, a_s, w, ws, K, out_min=-0.5, out_max=0.75)
    want = (ey + res).astype(np.float32)
    got = y.cpu().numpy()
    assert f32_bits_equal(got[:, 136:900], want[:, 136:900])
    assert np.isnan(got[:, :136]).all() and np.isnan(got[:, 900:]).all()
    assert int(wsp.abs().sum().item()) == 0


def test_stream_gemm_back_to_back_distinct_weights(e2c, of, torch_cuda):
    """A chain of launches over different weights on one stream and one workspace, with no
    synchronisation between them (the decode pattern the kernel exists for): every output
    bit-exact."""
    torch = torch_cuda
    rng = np.random.default_rng(91)
    M = 16
    outs = []
    for N, K in [(8192, 2048), (2048, 8192), (2048, 2048), (3072, 2048)]:
        qa, a_s, w, ws = _gemm_inputs(rng, M, N, K, K)
        W = e2c.Weight(w=w, scale=ws)
        y = e2c.i8_gemm(W, dev(torch, qa), dev(torch, a_s), K)
        outs.append((y, of.gemm_plain(qa, a_s, w, ws, K), W))
    e2c.check()
    for y, ey, _ in outs:
        assert f32_bits_equal(y.cpu().numpy(), ey)


# ------------------------------------------------------------------------------------------ GQA / vision attention
def _attn_ref_gqa(q, k, v, valid, B, S, H, KV, D, scale):
    """fp64 attention with KV heads (query head h reads KV head h // (H // KV)); invalid query rows 0."""
    out = np.zeros((B * S, H * D), np.float64)
    for b in range(B):
        keys = np.arange(S) if valid is None else np.nonzero(valid[b])[0]
        for h in range(H):
            kvh = h // (H // KV)
            if len(keys) == 0:
                continue
            qh = q[b * S:(b + 1) * S, h * D:(h + 1) * D].astype(np.float64)
            kb = k[b * S + keys, kvh * D:(kvh + 1) * D].astype(np.float64)
            vb = v[b * S + keys, kvh * D:(kvh + 1) * D].astype(np.float64)
            lg = qh @ kb.T * scale
            lg -= lg.max(axis=1, keepdims=True)
            pr = np.exp(lg)
            pr /= pr.sum(axis=1, keepdims=True)
            o = pr @ vb
            if valid is not None:
                o[valid[b] == 0] = 0
            out[b * S:(b + 1) * S, h * D:(h + 1) * D] = o
    return out


@pytest.mark.parametrize("B,S,H,KV,D,scale,masked", [
    (1, 2520, 12, 12, 64, 1.0, False),     # the vision tower: 2520 patches, 12 heads of 64, scale 1
    (2, 1000, 12, 12, 64, 0.125, True),    # fewer patches, masks, 1/sqrt(64)
    (3, 300, 12, 4, 64, 0.125, True),      # grouped KV heads at D = 64
    (2, 512, 4, 2, 256, 1 / 16, True),     # two KV heads at D = 256
    (1, 77, 2, 1, 64, 1.0, False),         # one partial tile
])
def test_attention_gqa_vs_fp64(e2c, of, torch_cuda, B, S, H, KV, D, scale, masked):
    """The attention kernel at head dim 64 (the vision tower's) and with several KV heads, against fp64
    of the same bf16 inputs, and against the checker's fp32 attention (e2o_attention_f32, restating
    e2.c src/text.c:702-741 and src/vision.c:540-571) for the first sequence."""
    torch = torch_cuda
    rng = np.random.default_rng(S * 13 + H + KV + D)
    qf = torch.from_numpy(rng.standard_normal((B * S, H * D)).astype(np.float32)).to(torch.bfloat16)
    kf = torch.from_numpy(rng.standard_normal((B * S, KV * D)).astype(np.float32)).to(torch.bfloat16)
    vf = torch.from_numpy(rng.standard_normal((B * S, KV * D)).astype(np.float32)).to(torch.bfloat16)
    valid = None
    if masked:
        valid = np.ones((B, S), np.uint8)
        valid[-1, S - S // 5:] = 0
        valid[0, 3:11] = 0
    ldvt = (S + 7) // 8 * 8
    vt = torch.zeros((B, KV * D, ldvt), dtype=torch.bfloat16)
    vt[:, :, :S] = vf.reshape(B, S, KV * D).transpose(1, 2)
    vd = None if valid is None else dev(torch, valid.reshape(-1))
    ctx = e2c.attention_gqa(qf.cuda(), kf.cuda(), vt.cuda(), vd, B, S, H, KV, D, scale)
    e2c.check()
    got = ctx.cpu().numpy()
    q32, k32, v32 = (t.float().numpy() for t in (qf, kf, vf))
    want = _attn_ref_gqa(q32, k32, v32, valid, B, S, H, KV, D, scale)
    for b in range(B):
        for h in range(H):
            rows = slice(b * S, (b + 1) * S)
            g = got[rows, h * D:(h + 1) * D]
            w = want[rows, h * D:(h + 1) * D]
            live = np.linalg.norm(w, axis=1) > 0
            if valid is not None:
                assert np.all(g[valid[b] == 0] == 0)
            err = np.linalg.norm(g[live] - w[live], axis=1) / np.linalg.norm(w[live], axis=1)
            assert err.max() < 1e-2, f"b={b} h={h} worst row rel err {err.max()}"
            assert cosine_rows(g[live], w[live]).min() > 0.9999
    # the checker's own fp32 attention on sequence 0
    want0 = np.zeros((S, H * D), np.float32)
    vb0 = None if valid is None else np.ascontiguousarray(valid[0])
    qb, kb, vb = (np.ascontiguousarray(t[:S]) for t in (q32, k32, v32))
    of.port().e2o_attention_f32(of.port().e2o_port_kernels(0), qb.ctypes.data_as(of.f32p), kb.ctypes.data_as(of.f32p),
                                vb.ctypes.data_as(of.f32p), want0.ctypes.data_as(of.f32p),
                                None if vb0 is None else vb0.ctypes.data_as(of.u8p), S, H, KV, D, scale)
    live = np.linalg.norm(want0, axis=1) > 0
    assert cosine_rows(got[:S][live], want0[live]).min() > 0.9999


@pytest.mark.parametrize("N,K", [(768, 768), (3072, 768), (768, 3072), (2304, 768)])
def test_gemm_vision_tower_shapes(e2c, of, syn, torch_cuda, N, K):
    """The vision tower's projections (e2.c src/vision.c: 2520 patches, hidden 768, MLP 3072; q|k|v
    concatenated) on the GEMM kernels, per-token scales, bit-exact to the reference fold."""
    torch = torch_cuda
    M = 2520
    rng = np.random.default_rng(N + K)
    x = syn.activations(rng, M, K)
    q, s = e2c.quantize_rows(dev(torch, x), K)
    wq, ws = syn.quantize_weight_rows((rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)))
    W = e2c.Weight(w=wq, scale=ws)
    y = e2c.i8_gemm(W, q, s, K).cpu().numpy()
    e2c.check()
    eq, es = of.quantize_signed(x, K)
    assert np.array_equal(q.cpu().numpy(), eq)
    assert f32_bits_equal(y, of.gemm_plain(eq, es, wq, ws, K))


# ------------------------------------------------------------------------------------------ per-128-block mode
def test_qkv_post_matches_port(e2c, of, torch_cuda):
    """Per-block mode's q|k|v finish (e2c_qkv_post): per-head RMSNorm, RoPE and bf16 out from the GEMM's
    fp32 output, against the port's e2o_rmsnorm + e2o_rope_rows (src/kernels.c:76-87,112-126)."""
    torch = torch_cuda
    rng = np.random.default_rng(33)
    B, S, H, Dh = 3, 200, 3, 256
    M = B * S
    y = rng.standard_normal((M, (H + 2) * Dh)).astype(np.float32) * 3
    qg = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    kg = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    cs = np.empty((S, Dh), np.float32)
    sn = np.empty((S, Dh), np.float32)
    of.port().e2o_rope_tables(cs.ctypes.data_as(of.f32p), sn.ctypes.data_as(of.f32p), S, Dh, 10000.0)
    ldrope, ldvt = S + 3, (S + 7) // 8 * 8
    cT = np.zeros((128, ldrope), np.float32)
    sT = np.zeros((128, ldrope), np.float32)
    cT[:, :S], sT[:, :S] = cs[:, :128].T, sn[:, :128].T
    Q = torch.zeros((M, H * Dh), dtype=torch.bfloat16, device="cuda")
    K = torch.zeros((M, Dh), dtype=torch.bfloat16, device="cuda")
    Vt = torch.zeros((B, Dh, ldvt), dtype=torch.bfloat16, device="cuda")
    yd, gq, gk, cd, sdn = (dev(torch, t) for t in (y, qg, kg, cT, sT))
    lib = e2c.lib()
    lib.e2c_qkv_post.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p,
                                 C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    assert lib.e2c_qkv_post(yd.data_ptr(), (H + 2) * Dh, H, gq.data_ptr(), gk.data_ptr(), 1e-6, cd.data_ptr(),
                            sdn.data_ptr(), ldrope, S, Q.data_ptr(), K.data_ptr(), Vt.data_ptr(), ldvt, M,
                            torch.cuda.current_stream().cuda_stream) == 0, lib.e2c_msg().decode()
    e2c.check()
    port = of.port()
    yy = y.reshape(M, H + 2, Dh)
    exp = np.empty_like(yy)
    for hd in range(H + 2):
        blk = np.ascontiguousarray(yy[:, hd])
        gamma = qg if hd < H else (kg if hd == H else None)
        port.e2o_rmsnorm(blk.ctypes.data_as(of.f32p), M, Dh, None if gamma is None else gamma.ctypes.data_as(of.f32p), 1e-6)
        if hd <= H:
            port.e2o_rope_rows(blk.ctypes.data_as(of.f32p), 0, M, 1, Dh, Dh,
                               np.ascontiguousarray(np.tile(cs, (B, 1))).ctypes.data_as(of.f32p),
                               np.ascontiguousarray(np.tile(sn, (B, 1))).ctypes.data_as(of.f32p))
        exp[:, hd] = blk
    to_bf = lambda t: t.float().cpu().numpy()
    got = np.concatenate([to_bf(Q).reshape(M, H, Dh), to_bf(K).reshape(M, 1, Dh),
                          to_bf(Vt)[:, :, :S].transpose(0, 2, 1).reshape(M, 1, Dh)], axis=1)
    want = torch.from_numpy(exp).to(torch.bfloat16).float().numpy()
    diff = np.abs(got - want)
    tol = np.abs(want) * 2.0 ** -7 + 4e-6  # one bf16 ulp (the norm's sum order differs from the port's)
    assert np.all(diff <= tol), f"beyond one bf16 ulp: {int((diff > tol).sum())}, worst {diff.max()}"
    assert (diff == 0).mean() > 0.99


@pytest.mark.parametrize("ablk", [1152, 128])
def test_gelu_mul_quant(e2c, of, torch_cuda, ablk):
    """Per-block mode's gate|up finish (e2c_gelu_mul_quant): h = gelu_tanh(g) * u from the GEMM's fp32
    output (columns interleaved per 128), quantised per token or per 128-block. Per token it must give
    the bytes and scales of the fused gate|up + GELU + quantise kernel bit for bit; per block, the
    port's GELU and quantiser within the tie rule."""
    torch = torch_cuda
    rng = np.random.default_rng(35)
    M, D, I = 300, 768, 1152
    qa, a_s, w, ws = _gemm_inputs(rng, M, 2 * I, D, D)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    y = torch.empty((M, 2 * I), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, D)
    a.epi, a.y, a.ldy = e2c.EPI_F32, y.data_ptr(), 2 * I
    _launch(e2c, a, torch)
    q = torch.zeros((M, I), dtype=torch.int8, device="cuda")
    qs = torch.zeros((M, I // ablk), dtype=torch.float32, device="cuda")
    lib = e2c.lib()
    lib.e2c_gelu_mul_quant.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    assert lib.e2c_gelu_mul_quant(y.data_ptr(), 2 * I, I, q.data_ptr(), qs.data_ptr(), M, ablk,
                                  torch.cuda.current_stream().cuda_stream) == 0, lib.e2c_msg().decode()
    e2c.check()
    if ablk == I and lib.e2c_gemm_gelu_quant_supported(I // 128):
        qf = torch.zeros((M, I), dtype=torch.int8, device="cuda")
        qsf = torch.zeros((M,), dtype=torch.float32, device="cuda")
        a2 = _args_for(W, qd, sd, M, D)
        a2.epi, a2.q8, a2.ldq, a2.q8_scale = e2c.EPI_GELUQ, qf.data_ptr(), I, qsf.data_ptr()
        _launch(e2c, a2, torch)
        assert torch.equal(q, qf), "bytes differ from the fused gate|up + GELU + quantise kernel"
        assert np.array_equal(qs.cpu().numpy()[:, 0].view(np.int32), qsf.cpu().numpy().view(np.int32))
    yh = y.cpu().numpy().reshape(M, I // 128, 2, 128)
    g, u = np.ascontiguousarray(yh[:, :, 0].reshape(M, I)), np.ascontiguousarray(yh[:, :, 1].reshape(M, I))
    of.port().e2o_gelu_tanh(g.ctypes.data_as(of.f32p), g.size)
    h = (g * u).astype(np.float32)
    eq, es = of.quantize_signed(h, ablk)
    np.testing.assert_allclose(qs.cpu().numpy(), es, rtol=1e-5)
    pre = h.reshape(M, I // ablk, ablk) * (np.float32(127.0) / np.abs(h.reshape(M, I // ablk, ablk)).max(axis=2, keepdims=True))
    tie_tolerant_bytes(q.cpu().numpy(), eq, pre.reshape(M, I))


@pytest.mark.parametrize("M,K,I", [(300, 768, 1152), (4096, 512, 2048), (2176, 768, 1152), (129, 1024, 256),
                                   (1000, 256, 128)])
def test_gelu_quant_epilogue_per_block(e2c, of, torch_cuda, M, K, I):
    """Per-block mode's gate|up GEMM with GELU-gate and the per-128-block quantiser of h in its
    epilogue (the text tower's and the per-block encoder's FFN, e2.c src/text.c:950-953 with
    src/int8.c:178-209 per block): the int8 rows and scales are bit-identical to the per-block F32
    GEMM followed by e2c_gelu_mul_quant (both checked against the port above). 4096 and 2176 rows
    take the CTA-pair kernel (2176: a half-empty last pair), the others single CTAs."""
    torch = torch_cuda
    rng = np.random.default_rng(57 + M + K + I)
    qa, a_s, w, ws = _gemm_inputs(rng, M, 2 * I, K, 128)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = dev(torch, qa), dev(torch, a_s)
    y = torch.empty((M, 2 * I), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, K)
    a.ablk, a.epi, a.y, a.ldy = 128, e2c.EPI_F32, y.data_ptr(), 2 * I
    _launch(e2c, a, torch)
    want_q = torch.zeros((M, I), dtype=torch.int8, device="cuda")
    want_s = torch.zeros((M, I // 128), dtype=torch.float32, device="cuda")
    lib = e2c.lib()
    lib.e2c_gelu_mul_quant.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    assert lib.e2c_gelu_mul_quant(y.data_ptr(), 2 * I, I, want_q.data_ptr(), want_s.data_ptr(), M, 128,
                                  torch.cuda.current_stream().cuda_stream) == 0, lib.e2c_msg().decode()
    e2c.check()
    ldq = I + 16  # a row stride wider than the row
    q = torch.full((M, ldq), 99, dtype=torch.int8, device="cuda")
    s = torch.zeros((M, I // 128), dtype=torch.float32, device="cuda")
    a = _args_for(W, qd, sd, M, K)
    a.ablk, a.epi, a.q8, a.ldq, a.q8_scale = 128, e2c.EPI_GELUQ, q.data_ptr(), ldq, s.data_ptr()
    _launch(e2c, a, torch)
    qn = q.cpu().numpy()
    assert np.array_equal(qn[:, :I], want_q.cpu().numpy()), "bytes differ from the two-kernel path"
    assert np.all(qn[:, I:] == 99), "wrote past the row"
    assert f32_bits_equal(s.cpu().numpy(), want_s.cpu().numpy())


def test_fused_per_block_epilogues_reject_bad_arguments(e2c, torch_cuda):
    """The per-block fused epilogues refuse, before anything is launched, what they cannot compute:
    activation blocks other than 128 (the output quantiser's block is the CTA's 128 columns), gate|up
    rows not in groups of 256 from row 0, int8 rows not 16-byte aligned, q|k|v columns that are not
    nq q heads then equal k and v heads of 256, M not a multiple of seq_len, and norm forms without
    their outputs. Each returns -1 with a message naming the epilogue."""
    torch = torch_cuda
    lib = e2c.lib()
    lib.e2c_msg.restype = C.c_char_p
    rng = np.random.default_rng(3)
    M, K = 256, 512

    def args(N, ablk):
        W = e2c.Weight(w=rng.integers(-127, 128, size=(N, K), dtype=np.int8),
                       scale=rng.uniform(1e-4, 0.02, size=N).astype(np.float32))
        qa = torch.zeros((M, K), dtype=torch.int8, device="cuda")
        qs = torch.ones((M, K // ablk), dtype=torch.float32, device="cuda")
        a = e2c.gemm_args(W, qa, qs, M)
        a.ablk = ablk
        return a, [W, qa, qs]

    def rejected(a, what):
        rc = lib.e2c_gemm(C.byref(a), torch.cuda.current_stream().cuda_stream)
        msg = lib.e2c_msg().decode()
        assert rc == -1 and what in msg, (rc, msg)

    q8 = torch.zeros((M, 1040), dtype=torch.int8, device="cuda")
    q8s = torch.zeros((M, 8), dtype=torch.float32, device="cuda")
    # GELU-quantise, per block: a 256-wide activation block; an odd int8 row stride
    a, keep = args(512, 256)
    a.epi, a.q8, a.ldq, a.q8_scale = e2c.EPI_GELUQ, q8.data_ptr(), 256, q8s.data_ptr()
    rejected(a, "GELU-quantise")
    a, keep = args(512, 128)
    a.epi, a.q8, a.ldq, a.q8_scale = e2c.EPI_GELUQ, q8.data_ptr(), 264, q8s.data_ptr()
    rejected(a, "GELU-quantise")
    # q|k|v, per block: per-token scales; 3 q heads with unequal k and v heads; M not a multiple of S
    out = torch.zeros((M, 2048), dtype=torch.bfloat16, device="cuda")
    tab = torch.zeros((512, 128), dtype=torch.float32, device="cuda")
    for N, ablk, S in ((5 * 256, K, 128), (6 * 256, 128, 128), (5 * 256, 128, 100)):
        a, keep = args(N, ablk)
        a.epi, a.nq, a.seq_len, a.ldvt, a.ldrope = e2c.EPI_QKVPB, 3, S, 256, 128
        a.q_out = a.k_out = a.vt_out = out.data_ptr()
        a.rope_cos = a.rope_sin = tab.data_ptr()
        rejected(a, "q|k|v")
    # residual norms, per block: a 256-wide activation block; neither int8 rows nor a final gain
    res = torch.zeros((M, 512), dtype=torch.float32, device="cuda")
    g = torch.ones(512, device="cuda")
    for ablk, with_q8 in ((256, True), (128, False)):
        a, keep = args(512, ablk)
        a.epi, a.res, a.ldres, a.norm_g1, a.eps = e2c.EPI_NORMADD, res.data_ptr(), 512, g.data_ptr(), 1e-6
        if with_q8:
            a.q8, a.ldq, a.q8_scale = q8.data_ptr(), 512, q8s.data_ptr()
        rejected(a, "norm epilogue")
    e2c.check()
