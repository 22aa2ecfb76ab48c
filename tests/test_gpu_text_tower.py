"""e2.c's own text tower (EmbeddingGemma-2, src/text.c:924-984) on the device against e2.c's own
engine running the same checkpoint on the host (oracle/_ref/libe2ref_text.so).

The device path computes attention in bf16 on the tensor cores; e2.c computes it in fp32 below 128
keys and in int8 from 128 keys (its dispatch table), and its fp32 attention can be forced. Both sides
re-quantise every activation row to int8 before each GEMM, which makes 24 layers sensitive to the
last bit of their inputs, so the pooled embeddings differ by noise that averages over a sequence's
tokens: (1 - cosine) x valid tokens is about constant across sequences of any length. The gate is
e2.c's own: for every sequence, (1 - cos(device, e2.c fp32 attention)) x valid tokens must not exceed
the largest (1 - cos(e2.c int8 attention, e2.c fp32 attention)) x tokens that e2.c's own int8
attention shows on full 512-token sequences, measured in the same run. The kernels below the tower
are checked on their own against fp64 and the port.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import cosine_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tm(e2c):
    import e2c_b200.text_model as m

    return m


@pytest.fixture(scope="module")
def tower(e2c, tm, text_tensors, torch_cuda):
    w = tm.TextWeights(text_tensors)
    t = e2c.TextTower(w.desc(), max_tokens=8 * 2048, keepalive=w)
    yield t
    t.close()


def _valid_patterns(B: int, S: int) -> np.ndarray:
    """full, trailing padding, holes, all invalid, a short prefix; the rest full"""
    v = np.ones((B, S), np.uint8)
    v[1, S - S // 5:] = 0
    v[2, 10:40] = 0
    v[2, S // 2:S // 2 + 11] = 0
    v[3, :] = 0
    v[4, 33:] = 0
    return v


@pytest.fixture(scope="module")
def i8_budget(tm, ref_text):
    """(1 - cosine) x tokens of e2.c's int8 attention against its fp32 attention, worst of four full
    512-token sequences: the per-token error e2.c accepts from its own default attention path."""
    ids = tm.token_ids(np.random.default_rng(4096), 4, 512)
    c = cosine_rows(ref_text.embed_batch(ids), ref_text.embed_batch(ids, attention=0))
    budget = float(((1.0 - c) * 512).max())
    print(f"\ne2.c int8 vs fp32 attention at 512 tokens: cos {c}, budget {budget:.4f}")
    assert 0 < budget < 2.0
    return budget


def _gate(got, want, valid, budget):
    n = valid.astype(np.int64).sum(axis=1)
    live = n > 0
    c = cosine_rows(got[live], want[live])
    per_token = (1.0 - c) * n[live]
    print(f"\ncos(device, e2.c fp32 attention) {np.round(c, 6)}; (1 - cos) x tokens {np.round(per_token, 4)}, "
          f"budget {budget:.4f}")
    assert np.all(got[~live] == 0) and np.all(want[~live] == 0)
    assert np.all(per_token <= budget), (per_token, budget)
    # an absolute floor where the noise has tokens to average over (a single token's embedding
    # differs from e2.c's by 1 - cos of about 0.05, as the per-token figure says)
    assert np.all(c[n[live] >= 64] > 0.99), c


def test_text_tower_vs_reference_512(tm, tower, ref_text, i8_budget):
    """8 sequences of 512 tokens with padding, holes, an all-invalid sequence and a short prefix."""
    rng = np.random.default_rng(512)
    B, S = 8, 512
    ids = tm.token_ids(rng, B, S)
    valid = _valid_patterns(B, S)
    got = tower.embed_batch(ids, valid)
    f32 = ref_text.embed_batch(ids, valid, attention=0)
    _gate(got, f32, valid, i8_budget)
    assert np.allclose(np.linalg.norm(got[np.arange(B) != 3], axis=1), 1.0, atol=1e-5)


def test_text_tower_vs_reference_sliding_window(tm, tower, ref_text, i8_budget):
    """Sequences longer than the window (1536 tokens: keys beyond 512 positions are masked on the
    sliding layers), one with trailing padding."""
    rng = np.random.default_rng(1536)
    B, S = 2, 1536
    ids = tm.token_ids(rng, B, S)
    valid = np.ones((B, S), np.uint8)
    valid[1, 1200:] = 0
    got = tower.embed_batch(ids, valid)
    f32 = ref_text.embed_batch(ids, valid, attention=0)
    _gate(got, f32, valid, i8_budget)


def test_text_tower_short_sequences(tm, tower, ref_text, i8_budget):
    """Below 128 keys e2.c's own attention is fp32 (its dispatch table): 3 x 77 tokens, unmasked."""
    rng = np.random.default_rng(77)
    ids = tm.token_ids(rng, 3, 77)
    got = tower.embed_batch(ids)
    want = ref_text.embed_batch(ids)
    _gate(got, want, np.ones(ids.shape, np.uint8), i8_budget)
    one = tower.embed(ids[1])
    assert np.array_equal(one, got[1])  # e2cuda_text_embed is the batch of one


def test_description_from_reference_loader_gives_identical_results(e2c, tm, tower, ref_text):
    """The tower built from the description e2.c's binding fills from its e2_model, and through the
    binding's own entry points (e2_cuda_create / e2_cuda_text_embed_batch), returns the same bits as
    the tower built from the package's quantisation of the same checkpoint."""
    layers = (tm.TextLayer * 24)()
    d = tm.TextDesc()
    ref_text.describe(d, layers)
    t2 = e2c.TextTower(d, max_tokens=4 * 512, keepalive=layers)
    rng = np.random.default_rng(11)
    ids = tm.token_ids(rng, 4, 300)
    valid = np.ones((4, 300), np.uint8)
    valid[2, 250:] = 0
    a = tower.embed_batch(ids, valid)
    b = t2.embed_batch(ids, valid)
    t2.close()
    c = ref_text.cuda_embed_batch(ids, valid)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def test_text_tower_short_and_odd_lengths(tm, tower, ref_text, i8_budget):
    """One token, and odd lengths that end mid-tile (e2_hip_text_embed takes any n_ids <= 2048)."""
    rng = np.random.default_rng(13)
    for S in (1, 13, 129):
        ids = tm.token_ids(rng, 2, S)
        got = tower.embed_batch(ids)
        want = ref_text.embed_batch(ids, attention=0)
        _gate(got, want, np.ones(ids.shape, np.uint8), i8_budget)


def test_text_tower_chunks_whole_sequences(e2c, tm, tower, text_tensors):
    """A tower whose device pass holds 3 sequences of 300 tokens embeds 5 in two passes, with the
    same bits as one pass over all 5 (rows never mix across sequences)."""
    w = tm.TextWeights(text_tensors)
    small = e2c.TextTower(w.desc(), max_tokens=1000, keepalive=w)
    rng = np.random.default_rng(300)
    ids = tm.token_ids(rng, 5, 300)
    valid = np.ones((5, 300), np.uint8)
    valid[3, 200:] = 0
    a = small.embed_batch(ids, valid)
    calls, _, _ = small.stats()
    small.close()
    b = tower.embed_batch(ids, valid)
    assert calls == 1
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_text_tower_rejects_bad_ids(e2c, tm, tower):
    """A token id outside the vocabulary fails the call before any device work (src/text.c:1005-1011)."""
    ids = tm.token_ids(np.random.default_rng(1), 1, 16)
    ids[0, 7] = 262144
    with pytest.raises(e2c.E2CudaError, match="out of range"):
        tower.embed_batch(ids)


def test_text_tower_graph_replay_and_stats(tm, tower):
    """The second call of a shape replays the captured graph and gives the same bits."""
    rng = np.random.default_rng(5)
    ids = tm.token_ids(rng, 2, 256)
    a = tower.embed_batch(ids)
    b = tower.embed_batch(ids)
    assert np.array_equal(a, b)
    calls, kernels, ms = tower.stats()
    # 14 kernels per layer, less gate|up's GELU-quantise epilogue, the three residual norms in the
    # o_proj, down and PLE-projection epilogues (every layer) and the q|k|v finish in the q|k|v
    # GEMM's epilogue (the 20 sliding layers, heads of 256)
    assert kernels == 5 + 9 * 20 + 10 * 4 and calls >= 2 and ms > 0


# ------------------------------------------------------------------------------ kernels of the tower
def _attn_fp64(q, k, v, valid, B, S, H, KV, D, window):
    out = np.zeros((B * S, H * D), np.float64)
    idx = np.arange(S)
    for b in range(B):
        vb = np.ones(S, bool) if valid is None else valid[b].astype(bool)
        keep = vb[None, :] & (np.abs(idx[:, None] - idx[None, :]) <= (window if window >= 0 else S))
        for h in range(H):
            kvh = h // (H // KV)
            qh = q[b * S:(b + 1) * S, h * D:(h + 1) * D].astype(np.float64)
            kh = k[b * S:(b + 1) * S, kvh * D:(kvh + 1) * D].astype(np.float64)
            vh = v[b * S:(b + 1) * S, kvh * D:(kvh + 1) * D].astype(np.float64)
            lg = np.where(keep, qh @ kh.T, -np.inf)
            m = lg.max(axis=1, keepdims=True)
            m[~np.isfinite(m)] = 0
            p = np.exp(lg - m)
            s = p.sum(axis=1, keepdims=True)
            o = np.where(s > 0, (p @ vh) / np.where(s > 0, s, 1), 0)
            o[~vb] = 0
            out[b * S:(b + 1) * S, h * D:(h + 1) * D] = o
    return out


@pytest.mark.parametrize("B,S,H,KV,D,window,masked", [
    (2, 512, 4, 1, 512, -1, True),    # the full-attention layers: head dim 512, one KV head
    (1, 700, 4, 1, 512, -1, False),   # a partial query tile and key tile
    (2, 1100, 4, 2, 256, 512, True),  # the sliding layers past the window
    (1, 300, 4, 2, 256, 40, False),   # a narrow window: most tiles cut by its edges
    (1, 600, 4, 1, 512, 100, True),   # the wide kernel with a window
])
def test_attention_window_vs_fp64(e2c, torch_cuda, B, S, H, KV, D, window, masked):
    torch = torch_cuda
    rng = np.random.default_rng(S + D + H + KV + window)
    # logits of sd ~ 1.4: unit-RMS rows (as after q/k RMSNorm) with gains 0.25, the checkpoint's tempering
    qf = torch.from_numpy((rng.standard_normal((B * S, H * D)) * 0.25).astype(np.float32)).to(torch.bfloat16)
    kf = torch.from_numpy((rng.standard_normal((B * S, KV * D)) * 0.25).astype(np.float32)).to(torch.bfloat16)
    vf = torch.from_numpy(rng.standard_normal((B * S, KV * D)).astype(np.float32)).to(torch.bfloat16)
    valid = None
    if masked:
        valid = np.ones((B, S), np.uint8)
        valid[-1, S - S // 4:] = 0
        valid[0, 5:30] = 0
    ldvt = (S + 7) // 8 * 8
    vt = torch.zeros((B, KV * D, ldvt), dtype=torch.bfloat16)
    vt[:, :, :S] = vf.reshape(B, S, KV * D).transpose(1, 2)
    vd = None if valid is None else torch.from_numpy(valid.reshape(-1)).cuda()
    ctx = e2c.attention_window(qf.cuda(), kf.cuda(), vt.cuda(), vd, B, S, H, KV, D, 1.0, window)
    e2c.check()
    got = ctx.cpu().numpy()
    want = _attn_fp64(*(t.float().numpy() for t in (qf, kf, vf)), valid, B, S, H, KV, D, window)
    live = np.linalg.norm(want.reshape(B * S * H, D), axis=1) > 0
    g, w = got.reshape(B * S * H, D), want.reshape(B * S * H, D)
    assert np.all(g[~live] == 0)
    err = np.linalg.norm(g[live] - w[live], axis=1) / np.linalg.norm(w[live], axis=1)
    assert err.max() < 1.5e-2, err.max()
    assert cosine_rows(g[live], w[live]).min() > 0.9999


@pytest.mark.parametrize("D,KV", [(512, 1), (256, 2)])
def test_tt_qkv_post_matches_port(e2c, of, torch_cuda, D, KV):
    """q|k|v finish of the tower's layers (e2c_tt_qkv_post): per-head RMSNorm (v without a gain),
    RoPE on q and k, bf16 Q, K, V^T, against the port's e2o_rmsnorm + e2o_rope_rows."""
    torch = torch_cuda
    rng = np.random.default_rng(D + KV)
    B, S, H = 2, 130, 4
    M = B * S
    nh = H + 2 * KV
    y = rng.standard_normal((M, nh * D)).astype(np.float32) * 3
    qg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    cs = np.empty((S, D), np.float32)
    sn = np.empty((S, D), np.float32)
    theta = 1e6 if D == 512 else 1e4
    of.port().e2o_rope_tables(cs.ctypes.data_as(of.f32p), sn.ctypes.data_as(of.f32p), S, D, theta)
    # the tower's position-major tables [pos][ldrope] (row padding 4 floats)
    ldrope, ldvt = D // 2 + 4, (S + 7) // 8 * 8
    cT = np.zeros((S, ldrope), np.float32)
    sT = np.zeros((S, ldrope), np.float32)
    cT[:, :D // 2], sT[:, :D // 2] = cs[:, :D // 2], sn[:, :D // 2]
    Q = torch.zeros((M, H * D), dtype=torch.bfloat16, device="cuda")
    K = torch.zeros((M, KV * D), dtype=torch.bfloat16, device="cuda")
    Vt = torch.zeros((B, KV * D, ldvt), dtype=torch.bfloat16, device="cuda")
    yd, gq, gk, cd, sdn = (torch.from_numpy(t).cuda() for t in (y, qg, kg, cT, sT))
    lib = e2c.lib()
    lib.e2c_tt_qkv_post.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_float,
                                    C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_int, C.c_int, C.c_void_p]
    assert lib.e2c_tt_qkv_post(yd.data_ptr(), nh * D, H, KV, D, gq.data_ptr(), gk.data_ptr(), 1e-6, cd.data_ptr(),
                               sdn.data_ptr(), ldrope, 1, S, Q.data_ptr(), K.data_ptr(), Vt.data_ptr(), ldvt, M,
                               torch.cuda.current_stream().cuda_stream) == 0, lib.e2c_msg().decode()
    e2c.check()
    port = of.port()
    yy = y.reshape(M, nh, D)
    exp = np.empty_like(yy)
    for hd in range(nh):
        blk = np.ascontiguousarray(yy[:, hd])
        gamma = qg if hd < H else (kg if hd < H + KV else None)
        port.e2o_rmsnorm(blk.ctypes.data_as(of.f32p), M, D, None if gamma is None else gamma.ctypes.data_as(of.f32p), 1e-6)
        if hd < H + KV:
            port.e2o_rope_rows(blk.ctypes.data_as(of.f32p), 0, M, 1, D, D,
                               np.ascontiguousarray(np.tile(cs, (B, 1))).ctypes.data_as(of.f32p),
                               np.ascontiguousarray(np.tile(sn, (B, 1))).ctypes.data_as(of.f32p))
        exp[:, hd] = blk
    f = lambda t: t.float().cpu().numpy()
    got = np.concatenate([f(Q).reshape(M, H, D), f(K).reshape(M, KV, D),
                          f(Vt)[:, :, :S].reshape(B, KV, D, S).transpose(0, 3, 1, 2).reshape(M, KV, D)], axis=1)
    want = torch.from_numpy(exp).to(torch.bfloat16).float().numpy()
    diff = np.abs(got - want)
    tol = np.abs(want) * 2.0 ** -7 + 4e-6
    assert np.all(diff <= tol), f"beyond one bf16 ulp: {int((diff > tol).sum())}, worst {diff.max()}"
    assert (diff == 0).mean() > 0.99


@pytest.mark.parametrize("B,S,H,KV,K", [(2, 512, 4, 2, 512), (16, 256, 4, 2, 512), (3, 77, 4, 2, 512),
                                        (4, 200, 3, 1, 768)])
def test_qkv_per_block_epilogue_matches_two_kernel_path(e2c, of, torch_cuda, B, S, H, KV, K):
    """The per-block q|k|v GEMM with the finish in its epilogue (E2C_EPI_QKVPB: per-head RMSNorm, v
    without a gain, RoPE from position-major tables, bf16 Q, K, V^T) against the per-block F32 GEMM
    followed by e2c_tt_qkv_post (checked against the port above). The fold and every element
    operation are the same; the norm's sum of squares is taken in another order, so values agree
    within one bf16 ulp and nearly all bit for bit. 16 x 256 rows take CTA pairs, 3 x 77 a ragged
    last tile; 4 x 200 is the synthetic encoder's 3 q heads and one KV head at K = 768."""
    torch = torch_cuda
    rng = np.random.default_rng(B * S + H + 7 * KV)
    D = 256
    M, nh = B * S, H + 2 * KV
    N = nh * D
    qa = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    a_s = rng.uniform(1e-3, 0.05, size=(M, K // 128)).astype(np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.uniform(1e-4, 0.02, size=N).astype(np.float32)
    W = e2c.Weight(w=w, scale=ws)
    qd, sd = torch.from_numpy(qa).cuda(), torch.from_numpy(a_s).cuda()
    qg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    cs = np.empty((S, D), np.float32)
    sn = np.empty((S, D), np.float32)
    of.port().e2o_rope_tables(cs.ctypes.data_as(of.f32p), sn.ctypes.data_as(of.f32p), S, D, 1e4)
    ldrope, ldvt = D // 2 + 4, (S + 7) // 8 * 8
    cT = np.zeros((S, ldrope), np.float32)
    sT = np.zeros((S, ldrope), np.float32)
    cT[:, :D // 2], sT[:, :D // 2] = cs[:, :D // 2], sn[:, :D // 2]
    gq, gk, cd, sdn = (torch.from_numpy(t).cuda() for t in (qg, kg, cT, sT))
    stream = torch.cuda.current_stream().cuda_stream

    def outputs():
        return (torch.zeros((M, H * D), dtype=torch.bfloat16, device="cuda"),
                torch.zeros((M, KV * D), dtype=torch.bfloat16, device="cuda"),
                torch.zeros((B, KV * D, ldvt), dtype=torch.bfloat16, device="cuda"))

    # two kernels: the per-block F32 GEMM, then the finish
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    a = e2c.gemm_args(W, qd, sd, M)
    a.ablk, a.epi, a.y, a.ldy = 128, e2c.EPI_F32, y.data_ptr(), N
    e2c.gemm_raw(a)
    Q0, K0, V0 = outputs()
    lib = e2c.lib()
    lib.e2c_tt_qkv_post.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_float,
                                    C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_int, C.c_int, C.c_void_p]
    assert lib.e2c_tt_qkv_post(y.data_ptr(), N, H, KV, D, gq.data_ptr(), gk.data_ptr(), 1e-6, cd.data_ptr(),
                               sdn.data_ptr(), ldrope, 1, S, Q0.data_ptr(), K0.data_ptr(), V0.data_ptr(), ldvt, M,
                               stream) == 0, lib.e2c_msg().decode()
    # one kernel
    Q1, K1, V1 = outputs()
    a = e2c.gemm_args(W, qd, sd, M)
    a.ablk, a.epi, a.nq = 128, e2c.EPI_QKVPB, H
    a.q_out, a.k_out, a.vt_out, a.ldvt, a.seq_len = Q1.data_ptr(), K1.data_ptr(), V1.data_ptr(), ldvt, S
    a.q_gamma, a.k_gamma, a.rope_cos, a.rope_sin = gq.data_ptr(), gk.data_ptr(), cd.data_ptr(), sdn.data_ptr()
    a.ldrope, a.eps = ldrope, 1e-6
    e2c.gemm_raw(a)
    e2c.check()
    f = lambda t: t.float().cpu().numpy()
    for got, want, what in ((Q1, Q0, "Q"), (K1, K0, "K"), (V1[:, :, :S], V0[:, :, :S], "V^T")):
        g, w_ = f(got), f(want)
        diff = np.abs(g - w_)
        tol = np.maximum(np.abs(g), np.abs(w_)) * 2.0 ** -7 + 1e-6
        assert np.all(diff <= tol), f"{what}: beyond one bf16 ulp: {int((diff > tol).sum())}, worst {diff.max()}"
        assert (diff == 0).mean() > 0.98, f"{what}: {(diff == 0).mean()} identical"
    assert torch.count_nonzero(V1[:, :, S:]) == 0, "V^T written past seq_len"
