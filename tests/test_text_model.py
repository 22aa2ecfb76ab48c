"""e2.c's own text tower without a GPU: the seeded checkpoint loads in e2.c's own loader, the
package quantises it to the same bytes the loader does, the description handed to the library
matches the one e2.c's binding fills from its e2_model, and e2.c's text tower embeds with it.
The device path is checked against this checker in test_gpu_text_tower.py."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest


@pytest.fixture(scope="module")
def tm(e2c):
    import e2c_b200.text_model as m

    return m


def test_description_layout_matches_the_library(e2c, tm):
    lib = C.CDLL(str(e2c.LIB_PATH))
    d, l = C.c_int(), C.c_int()
    lib.e2c_text_struct_sizes(C.byref(d), C.byref(l))
    assert (d.value, l.value) == (C.sizeof(tm.TextDesc), C.sizeof(tm.TextLayer))


def test_checkpoint_round_trip(tm, text_tensors, text_model_dir):
    back = tm.read_safetensors(text_model_dir / "model.safetensors")
    shapes = tm.tensor_shapes(tm.TextConfig())
    assert set(back) == set(shapes) == set(text_tensors)
    for name in ("language_model.layers.5.self_attn.q_proj.weight", "language_model.layers.0.layer_scalar",
                 "language_model.embed_tokens.weight"):
        assert back[name].shape == shapes[name]
        assert np.array_equal(back[name], text_tensors[name])


def test_quantisation_matches_the_reference_loader(e2c, tm, text_tensors, ref_text):
    """Every projection of the tower: the package's per-row quantiser + e2_q8w packing against the
    e2_q8w e2.c's loader built from the same checkpoint (src/int8.c:19-66,80-83), byte for byte
    (weights, block sums, scales), and the description's scalars and per-layer geometry."""
    ours = tm.TextWeights(text_tensors)
    layers = (tm.TextLayer * 24)()
    theirs = tm.TextDesc()
    ref_text.describe(theirs, layers)
    mine = ours.desc()
    for f, _ in tm.TextDesc._fields_[:12]:
        assert getattr(theirs, f) == getattr(mine, f), f

    def q8(addr):
        q = e2c.Q8W.from_address(addr)
        kq = (q.K + 3) // 4
        return (q.N, q.K, q.nblocks, np.ctypeslib.as_array(q.w, shape=(q.Npad * kq * 4,)).copy(),
                np.ctypeslib.as_array(q.scale, shape=(q.Npad,)).copy(),
                np.ctypeslib.as_array(q.bsq, shape=(q.nblocks * q.Npad,)).copy())

    def same(a, b):
        return a[:3] == b[:3] and all(np.array_equal(x, y) for x, y in zip(a[3:], b[3:]))

    for l in range(24):
        for k in ("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj"):
            assert same(q8(getattr(layers[l], k)), q8(getattr(ours.layers[l], k))), (l, k)
        for k in ("layer_scalar", "head_dim", "n_kv_heads", "window", "rope_theta"):
            assert getattr(layers[l], k) == getattr(ours.layers[l], k), (l, k)
        for k in ("input_ln", "q_norm"):
            n = layers[l].head_dim if k == "q_norm" else 512
            a = np.ctypeslib.as_array(C.cast(getattr(layers[l], k), C.POINTER(C.c_float)), shape=(n,))
            b = np.ctypeslib.as_array(C.cast(getattr(ours.layers[l], k), C.POINTER(C.c_float)), shape=(n,))
            assert np.array_equal(a, b), (l, k)
    for k in ("ple_model_proj", "embed_proj"):
        assert same(q8(getattr(theirs, k)), q8(getattr(mine, k))), k
    assert [layers[l].head_dim for l in range(24)] == [512 if l in tm.FULL_LAYERS else 256 for l in range(24)]


def test_reference_text_tower_embeds(tm, ref_text):
    """e2.c's text tower on the checkpoint: unit vectors, exact zeros for an all-invalid sequence,
    and a padded sequence equal to its unpadded self (positions restart per sequence)."""
    rng = np.random.default_rng(3)
    ids = tm.token_ids(rng, 3, 48)
    valid = np.ones((3, 48), np.uint8)
    valid[1, :] = 0
    valid[2, 40:] = 0
    out = ref_text.embed_batch(ids, valid)
    assert np.allclose(np.linalg.norm(out[[0, 2]], axis=1), 1.0, atol=1e-5)
    assert np.all(out[1] == 0)
    short = ref_text.embed_batch(ids[2:3, :40])
    cos = float(out[2] @ short[0])
    assert cos > 0.9999, cos


def test_text_create_rejects_bad_descriptions(e2c, tm, text_tensors):
    """Geometry is checked before any device work: a hidden size off the 128 grid, a layer whose
    head dim is neither 256 nor 512, a projection whose shape disagrees with the description, and an
    activation block other than 128 or hidden all fail with a message (no GPU needed)."""
    w = tm.TextWeights(text_tensors)
    lib = e2c.lib()

    def create(d):
        return lib.e2cuda_text_create(C.addressof(d), 1024)

    d = w.desc()
    d.hidden = 500
    assert create(d) is None and "unsupported geometry" in e2c.last_error()
    d = w.desc()
    d.ablk = 64
    assert create(d) is None and "ablk" in e2c.last_error()
    d = w.desc()
    saved = w.layers[3].head_dim
    w.layers[3].head_dim = 384
    try:
        assert create(d) is None and "layer 3" in e2c.last_error()
    finally:
        w.layers[3].head_dim = saved
    saved = w.layers[7].o
    w.layers[7].o = w.layers[7].q  # q is [1024][512], o must be [512][1024]
    try:
        assert create(w.desc()) is None and "layer 7" in e2c.last_error()
    finally:
        w.layers[7].o = saved
