"""Host-side logic that needs no GPU: the seeded synthetic configs and the numpy weight quantiser
that bench.py uses (pinned against the port, which tests/test_oracle.py pins against the
reference)."""
from __future__ import annotations

import numpy as np


def test_numpy_weight_quantiser_matches_port(of, syn):
    rng = np.random.default_rng(0)
    for N, K, blk in ((24, 256, 128), (40, 768, 768), (9, 1152, 128)):
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        w[2] = 0
        pw = syn.PackedWeight(*syn.quantize_weight_rows(w), blk)
        ow = of.Weight(w, blk)
        assert np.array_equal(pw.packed, ow.q.packed())
        assert np.array_equal(pw.scale_pad.view(np.int32), ow.q.scales().view(np.int32))
        assert np.array_equal(pw.bsq, ow.q.bsums())
        assert np.array_equal(ow.plain(), pw.q)


def test_config_generators(syn):
    rng = np.random.default_rng(1)
    x = syn.activations(rng, 512, 768)
    big = np.abs(x).mean(axis=0)
    assert all(big[c] > 10 * np.median(big) for c in syn.OUTLIER_CHANNELS)
    ids = syn.token_batch(rng, 64, 512, 262144)
    assert ids.min() >= 2 and ids.max() < 262144 and ids.dtype == np.int32
    lens = syn.log_uniform_lengths(rng, 65536)
    assert lens.min() >= 32 and lens.max() <= 2048
    assert 420 < lens.mean() < 550  # mean of floor(exp(U[ln 32, ln 2048])) is ~485


def test_encoder_weights_shapes(syn):
    cfg = syn.EncoderConfig(n_layers=2, vocab=512)
    w = syn.encoder_weights(cfg, seed=1)
    lay = w.layers[0]
    assert lay["wq"].q.shape == (768, 768) and lay["wk"].q.shape == (256, 768)
    assert lay["wg"].q.shape == (1152, 768) and lay["wd"].q.shape == (768, 1152)
    assert w.table.shape == (512, 768) and w.dense1.q.shape == (3072, 768) and w.dense2.q.shape == (768, 3072)
    assert abs(cfg.embed_scale - np.sqrt(768)) < 1e-4
