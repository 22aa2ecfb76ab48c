"""The CPU port (oracle/liboracle.so) against the golden fixtures that tests/golden/make_golden.py
produced by running the reference's own kernels. These hold wherever the tests run, with or
without the reference sources; together with tests/test_oracle.py they pin the checker that every
GPU parity test uses."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from conftest import cosine_rows

GOLDEN = Path(__file__).resolve().parent / "golden" / "int8_path.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


@pytest.mark.parametrize("tag", ["q128_768", "q768_768", "q1152_1152", "q128_512"])
def test_quantizer_fixture(of, gold, tag):
    blk = int(tag[1:].split("_")[0])
    x = gold[tag + "_x"]
    q, s = of.quantize_biased(x, blk)
    assert np.array_equal(q, gold[tag + "_q"])
    assert np.array_equal(s.view(np.int32), gold[tag + "_s"].view(np.int32))


def test_quantizer_clamp_fixture(of, gold):
    q, s = of.quantize_biased(gold["qclamp_x"], 128, -0.75, 0.5)
    assert np.array_equal(q, gold["qclamp_q"]) and np.array_equal(s, gold["qclamp_s"])


@pytest.mark.parametrize("blk", [128, 768, 1152])
def test_weight_pack_and_gemm_fixture(of, gold, blk):
    p = f"g{blk}_"
    w = of.Weight(gold[p + "w"], blk)
    assert np.array_equal(w.q.packed(), gold[p + "packed"])
    assert np.array_equal(w.q.scales().view(np.int32), gold[p + "scale"].view(np.int32))
    assert np.array_equal(w.q.bsums(), gold[p + "bsq"])
    qa, sa = gold[p + "qa"], gold[p + "sa"]
    M, N = gold[p + "y"].shape
    y = np.full((M, N), -7.0, np.float32)
    of.port().e2o_i8_gemm(y.ctypes.data_as(of.f32p), np.ascontiguousarray(qa).view(np.int8).ctypes.data_as(of.i8p),
                          np.ascontiguousarray(sa).ctypes.data_as(of.f32p), C.byref(w.q), M, N, 8, N - 3, blk)
    assert np.array_equal(y.view(np.int32), gold[p + "y"].view(np.int32))


def test_ffn_fixture(of, syn, gold):
    wg = syn.PackedWeight(gold["ffn_wg_q"], gold["ffn_wg_s"], 128)
    wu = syn.PackedWeight(gold["ffn_wu_q"], gold["ffn_wu_s"], 128)
    wd = syn.PackedWeight(gold["ffn_wd_q"], gold["ffn_wd_s"], 256)
    y, st = of.ffn_block("port", gold["ffn_x"], gold["ffn_g"], 1e-6, wg, wu, wd, ablk=0, stages=True)
    # the port's RMSNorm is IEEE; the reference's is -ffast-math: bytes may differ by
    # one step at a tie, outputs by a few ulp
    d = np.abs(st["xq"].astype(int) - gold["ffn_xq"].astype(int))
    assert d.max() <= 1 and (d == 0).mean() > 0.999
    err = np.linalg.norm(y - gold["ffn_y"], axis=1) / np.linalg.norm(gold["ffn_y"], axis=1)
    assert err.max() < 1e-4


def test_encoder_fixture(of, syn, gold):
    cfg = syn.EncoderConfig(n_layers=1, hidden=128, n_heads=2, head_dim=64, ffn=256, vocab=64, dense_hidden=256,
                            out_dim=128, max_seq=16)
    w = syn.encoder_weights(cfg, seed=int(gold["enc_seed"][0]))
    y = of.encoder_forward("port", w, gold["enc_ids"], gold["enc_valid"])
    assert cosine_rows(y, gold["enc_out"]).min() >= 0.9999
