"""Generate the golden fixtures of the int8 hot path from the reference itself.

Runs the reference e2.c kernels, compiled from their own sources by oracle/Makefile into
oracle/_ref/ (one library per activation block E2_I8_BLOCK), on seeded inputs, and stores inputs and
outputs under tests/golden/*.npz. The reference sources exist only on the build host, so the
fixtures are committed; tests/test_golden.py checks the CPU port (oracle/liboracle.so) against them
wherever it runs.

    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle_ffi as of  # noqa: E402

spec = importlib.util.spec_from_file_location("e2c_b200.synthetic", ROOT / "e2.c_b200" / "synthetic.py")
syn = importlib.util.module_from_spec(spec)
sys.modules["e2c_b200.synthetic"] = syn
spec.loader.exec_module(syn)


def quantizer(rng):
    out = {}
    for blk, M, K in ((128, 24, 768), (768, 24, 768), (1152, 8, 1152), (128, 8, 512)):
        lib = of.ref(blk)
        x = syn.activations(rng, M, K) * rng.uniform(1e-3, 10, (M, 1)).astype(np.float32)
        x = np.ascontiguousarray(x, np.float32)
        x[1] = 0
        x[3, :blk] = 0
        q, s = of.quantize_biased(x, blk, lib=lib, fn="e2_quantize_blocks_avx512")
        out[f"q{blk}_{K}_x"], out[f"q{blk}_{K}_q"], out[f"q{blk}_{K}_s"] = x, q, s
    # the clamped form the audio tower uses
    lib = of.ref(128)
    x = syn.activations(rng, 8, 256)
    q, s = of.quantize_biased(x, 128, -0.75, 0.5, lib=lib, fn="e2_quantize_blocks_avx512")
    out["qclamp_x"], out["qclamp_q"], out["qclamp_s"] = x, q, s
    return out


def weights_and_gemm(rng):
    out = {}
    for blk, M, N, K in ((128, 16, 72, 512), (768, 16, 64, 768), (1152, 9, 40, 1152)):
        lib = of.ref(blk)
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        w[5] = 0  # an all-zero row: scale 1
        qw = of.Weight(w, blk, lib)
        x = syn.activations(rng, M, K)
        qa, sa = of.quantize_biased(x, blk, lib=lib, fn="e2_quantize_blocks_avx512")
        y = np.full((M, N), -7.0, np.float32)
        lib.e2_i8_gemm_avx512(y.ctypes.data_as(of.f32p), qa.view(np.int8).ctypes.data_as(of.i8p),
                              sa.ctypes.data_as(of.f32p), C.byref(qw.q), M, N, 8, N - 3)
        p = f"g{blk}_"
        out.update({p + "w": w, p + "packed": qw.q.packed(), p + "scale": qw.q.scales(), p + "bsq": qw.q.bsums(),
                    p + "qa": qa, p + "sa": sa, p + "y": y})
    return out


def ffn(rng):
    M, D, I = 8, 128, 256
    x = rng.standard_normal((M, D), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wg, wu = syn.packed_weight(rng, I, D, 0.02, D), syn.packed_weight(rng, I, D, 0.02, D)
    wd = syn.packed_weight(rng, D, I, 0.02, I)
    y, st = of.ffn_block("reference", x, g, 1e-6, wg, wu, wd, ablk=0, stages=True)
    return {"ffn_x": x, "ffn_g": g, "ffn_wg_q": wg.q, "ffn_wg_s": wg.scale, "ffn_wu_q": wu.q, "ffn_wu_s": wu.scale,
            "ffn_wd_q": wd.q, "ffn_wd_s": wd.scale, "ffn_y": y, "ffn_xq": st["xq"], "ffn_hq": st["hq"]}


def encoder(rng):
    cfg = syn.EncoderConfig(n_layers=1, hidden=128, n_heads=2, head_dim=64, ffn=256, vocab=64, dense_hidden=256,
                            out_dim=128, max_seq=16)
    w = syn.encoder_weights(cfg, seed=11)
    ids = syn.token_batch(rng, 2, 16, cfg.vocab)
    valid = np.ones((2, 16), np.uint8)
    valid[1, 12:] = 0
    y = of.encoder_forward("reference", w, ids, valid)
    return {"enc_ids": ids, "enc_valid": valid, "enc_seed": np.array([11]), "enc_out": y}


def main():
    if of.mux() is None:
        sys.exit("reference builds missing: run make -C oracle with the reference sources present")
    rng = np.random.default_rng(0xE2C0DE)
    data = {}
    for part in (quantizer, weights_and_gemm, ffn, encoder):
        data.update(part(rng))
    np.savez_compressed(HERE / "int8_path.npz", **data)
    print(f"wrote {HERE / 'int8_path.npz'} ({(HERE / 'int8_path.npz').stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
