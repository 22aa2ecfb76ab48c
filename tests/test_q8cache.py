"""The .e8cq model cache (A11) without a GPU: the library's reader and writer against the
reference's own (e2.c src/q8cache.c, compiled from its sources into oracle/_ref) in both directions,
the kind-4 device-layout entry, conversion of a version-1 cache, and the reader's checks on
damaged files. The device upload is in test_gpu_kernels.py."""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import pytest

HDR = struct.Struct("<4I")
ENTRY = struct.Struct("<96sII4qQQ")  # name, kind, ndim, dims[4], nbytes, off: 152 bytes


def _weights(of, seed=5):
    """Two packed e2_q8w of block 128 (the reference's default build) with N not a multiple of 8."""
    rng = np.random.default_rng(seed)
    return {"model.layers.0.mlp.down_proj.weight": of.Weight(rng.standard_normal((77, 256)).astype(np.float32) * 0.02, 128),
            "model.layers.0.self_attn.q_proj.weight": of.Weight(rng.standard_normal((40, 384)).astype(np.float32), 128)}


def _dense(seed=6):
    rng = np.random.default_rng(seed)
    return {"model.norm.weight": (2, rng.standard_normal(96).astype(np.float32)),
            "model.embed_tokens.weight": (1, rng.integers(0, 65535, size=(33, 16), dtype=np.uint16)),
            "model.layers.0.mlp.down_proj.input_max": (2, np.array(3.5, np.float32)),  # rank 0: one element
            "empty": (2, np.zeros((0, 4), np.float32))}


def _index(path):
    b = path.read_bytes()
    magic, ver, n, off = HDR.unpack_from(b, 0)
    return magic, ver, [ENTRY.unpack_from(b, off + i * ENTRY.size) for i in range(n)]


def _ref_write(ref, path, weights, dense):
    assert ref.q8c_write_open(str(path).encode()) == 0, ref.q8c_error()
    keep = []
    for name, w in weights.items():
        assert ref.q8c_put_q8w(name.encode(), C.byref(w.q)) == 0, ref.q8c_error()
    for name, (kind, a) in dense.items():  # the reference writes deferred tensors at close, in order
        a = np.array(a, order="C")  # (np.ascontiguousarray would make a rank-0 tensor rank 1)
        dims = (C.c_int64 * 4)(*a.shape)
        keep.append((a, dims))
        assert ref.q8c_defer(name.encode(), kind, a.ndim, dims, a.ctypes.data_as(C.c_void_p), a.nbytes) == 0
    assert ref.q8c_write_close() == 0, ref.q8c_error()


def _our_write(e2c, path, weights, dense):
    w = e2c.Q8CacheWriter(path)
    for name, q in weights.items():
        w.put_q8w(name, q.q)
    for name, (kind, a) in dense.items():
        w.put(name, kind, a)
    w.commit()


@pytest.fixture
def ref(of):
    r = of.ref_q8cache()
    if r is None:
        pytest.skip("the reference's q8cache.c was not built here (oracle/_ref)")
    return r


def test_files_are_byte_identical_to_the_reference_writer(e2c, of, ref, tmp_path):
    weights, dense = _weights(of), _dense()
    _ref_write(ref, tmp_path / "ref.e8cq", weights, dense)
    _our_write(e2c, tmp_path / "ours.e8cq", weights, dense)
    a, b = (tmp_path / "ref.e8cq").read_bytes(), (tmp_path / "ours.e8cq").read_bytes()
    assert len(a) == len(b) and a == b
    assert _index(tmp_path / "ours.e8cq")[1] == 1


def test_reads_what_the_reference_writes(e2c, of, ref, tmp_path):
    weights, dense = _weights(of), _dense()
    _ref_write(ref, tmp_path / "ref.e8cq", weights, dense)
    c = e2c.Q8Cache(tmp_path / "ref.e8cq")
    assert c.version == 1
    ents = {n: (k, d, nb) for n, k, d, nb in c.entries()}
    assert set(ents) == set(weights) | set(dense)
    for name, w in weights.items():
        q = c.q8w(name)
        assert (q.N, q.K, q.nblocks, q.Npad) == (w.q.N, w.q.K, w.q.nblocks, w.q.Npad)
        assert q.borrowed == 1 and q.out_min == np.float32(-1e31) and q.out_max == np.float32(1e31)
        got = of.Q8W.from_buffer_copy(bytes(q))
        np.testing.assert_array_equal(got.packed(), w.q.packed())
        np.testing.assert_array_equal(got.scales(), w.q.scales())
        np.testing.assert_array_equal(got.bsums(), w.q.bsums())
    for name, (kind, a) in dense.items():
        assert ents[name][0] == kind and ents[name][1] == a.shape
        np.testing.assert_array_equal(c.blob(name, kind), np.frombuffer(a.tobytes(), np.uint8))
    c.close()


def test_the_reference_reads_what_we_write(e2c, of, ref, tmp_path):
    weights, dense = _weights(of), _dense()
    _our_write(e2c, tmp_path / "ours.e8cq", weights, dense)
    assert ref.q8c_read_open(str(tmp_path / "ours.e8cq").encode()) == 0, ref.q8c_error()
    try:
        for name, w in weights.items():
            q = of.Q8W()
            assert ref.q8c_get_q8w(name.encode(), C.byref(q)) == 0
            np.testing.assert_array_equal(q.packed(), w.q.packed())
            np.testing.assert_array_equal(q.bsums(), w.q.bsums())
        for name, (kind, a) in dense.items():
            n = C.c_size_t()
            dims = (C.c_int64 * 4)(*a.shape)
            p = ref.q8c_get(name.encode(), kind, a.ndim, dims, C.byref(n))
            assert p and n.value == a.nbytes
            if n.value:
                assert C.string_at(p, n.value) == a.tobytes()
    finally:
        ref.q8c_read_close()


def _tiled(w, rows, ld):
    t = np.zeros((rows, ld), np.int8)
    t[: w.N, : w.K] = w.plain()
    s = np.zeros(rows, np.float32)
    s[: w.N] = w.scales()
    return np.concatenate([t.view(np.uint8).ravel(), s.view(np.uint8)])


def test_kind4_holds_the_device_layout(e2c, of, tmp_path):
    weights = _weights(of)
    w = e2c.Q8CacheWriter(tmp_path / "v2.e8cq")
    for name, q in weights.items():
        w.put_w8(name, q.q)
    w.put("model.norm.weight", e2c.Q8C_F32, np.ones(8, np.float32))
    w.commit()
    c = e2c.Q8Cache(tmp_path / "v2.e8cq")
    assert c.version == 2
    ents = {n: (k, d, nb) for n, k, d, nb in c.entries()}
    for name, q in weights.items():
        rows, ld = (q.N + 15) // 16 * 16, (q.K + 15) // 16 * 16
        assert ents[name] == (e2c.Q8C_W8, (q.N, q.K, rows, ld), rows * ld + 4 * rows)
        np.testing.assert_array_equal(c.blob(name, e2c.Q8C_W8), _tiled(q, rows, ld))
        with pytest.raises(e2c.E2CudaError, match="kind"):
            c.q8w(name)  # a kind-4 entry is not an e2_q8w
    c.close()


def test_the_reference_refuses_version_2(e2c, of, ref, tmp_path):
    weights = _weights(of)
    w = e2c.Q8CacheWriter(tmp_path / "v2.e8cq")
    w.put_w8("w", weights["model.layers.0.mlp.down_proj.weight"].q)
    w.commit()
    assert ref.q8c_read_open(str(tmp_path / "v2.e8cq").encode()) != 0
    assert b"version" in ref.q8c_error()


def test_convert_rewrites_weights_as_kind4(e2c, of, ref, tmp_path):
    weights, dense = _weights(of), _dense()
    _ref_write(ref, tmp_path / "v1.e8cq", weights, dense)
    e2c.q8c_convert(tmp_path / "v1.e8cq", tmp_path / "v2.e8cq")
    a, b = e2c.Q8Cache(tmp_path / "v1.e8cq"), e2c.Q8Cache(tmp_path / "v2.e8cq")
    assert b.version == 2
    assert [n for n, *_ in a.entries()] == [n for n, *_ in b.entries()]
    for name, kind, dims, nb in b.entries():
        if name in weights:
            q = weights[name]
            assert kind == e2c.Q8C_W8
            np.testing.assert_array_equal(b.blob(name, kind), _tiled(q, dims[2], dims[3]))
        else:
            np.testing.assert_array_equal(b.blob(name, kind), a.blob(name, kind))
    a.close()
    b.close()
    # converting twice changes nothing
    e2c.q8c_convert(tmp_path / "v2.e8cq", tmp_path / "v2b.e8cq")
    assert (tmp_path / "v2.e8cq").read_bytes() == (tmp_path / "v2b.e8cq").read_bytes()


def _damage(path, fn):
    b = bytearray(path.read_bytes())
    fn(b)
    path.write_bytes(bytes(b))


@pytest.mark.parametrize("how,msg", [
    ("truncate", "index"), ("magic", "e8cq"), ("misalign", "index"), ("nbytes", "dims need"),
    ("kind", "kind"), ("kind4_v1", "kind"), ("name", "name"), ("offset", "data area"), ("dims", "packed weight"),
    ("short", "header"),
])
def test_reader_rejects_damaged_files(e2c, of, tmp_path, how, msg):
    weights, dense = _weights(of), _dense()
    p = tmp_path / "c.e8cq"
    _our_write(e2c, p, weights, dense)
    _, _, ents = _index(p)
    idx = HDR.unpack_from(p.read_bytes(), 0)[3]
    first = idx  # the first entry: a kind-3 weight

    def set_entry(b, field, value):
        e = list(ENTRY.unpack_from(b, first))
        e[field] = value
        ENTRY.pack_into(b, first, *e)

    if how == "truncate":
        _damage(p, lambda b: b.__delitem__(slice(len(b) - 10, len(b))))
    elif how == "magic":
        _damage(p, lambda b: b.__setitem__(slice(0, 4), b"XXXX"))
    elif how == "misalign":
        _damage(p, lambda b: struct.pack_into("<I", b, 12, idx + 4))
    elif how == "nbytes":
        _damage(p, lambda b: set_entry(b, 7, ents[0][7] - 16))
    elif how == "kind":
        _damage(p, lambda b: set_entry(b, 1, 9))
    elif how == "kind4_v1":
        _damage(p, lambda b: set_entry(b, 1, 4))
    elif how == "name":
        _damage(p, lambda b: set_entry(b, 0, b"n" * 96))
    elif how == "offset":
        _damage(p, lambda b: set_entry(b, 8, idx + 16))
    elif how == "dims":
        _damage(p, lambda b: set_entry(b, 5, 10**6))  # nblocks beyond K is no e2_q8w
    elif how == "short":
        p.write_bytes(b"E8CQ")
    with pytest.raises(e2c.E2CudaError) as ei:
        e2c.Q8Cache(p)
    assert msg in str(ei.value).lower()


def test_writer_abort_and_refusals_leave_files_alone(e2c, of, tmp_path):
    p = tmp_path / "keep.e8cq"
    _our_write(e2c, p, _weights(of), {})
    before = p.read_bytes()
    w = e2c.Q8CacheWriter(p)
    w.put("a", e2c.Q8C_F32, np.ones(4, np.float32))
    with pytest.raises(e2c.E2CudaError, match="already"):
        w.put("a", e2c.Q8C_F32, np.ones(4, np.float32))
    with pytest.raises(e2c.E2CudaError, match="longer"):
        w.put("x" * 96, e2c.Q8C_F32, np.ones(4, np.float32))
    with pytest.raises(e2c.E2CudaError):
        w.put("b", e2c.Q8C_Q8W, np.ones(4, np.float32))  # packed weights go through put_q8w / put_w8
    w.abort()
    assert p.read_bytes() == before
    assert sorted(x.name for x in tmp_path.iterdir()) == ["keep.e8cq"]  # no temporary file left


def test_empty_cache_round_trips(e2c, ref, tmp_path):
    w = e2c.Q8CacheWriter(tmp_path / "empty.e8cq")
    w.commit()
    c = e2c.Q8Cache(tmp_path / "empty.e8cq")
    assert c.version == 1 and c.entries() == []
    c.close()
    assert ref.q8c_read_open(str(tmp_path / "empty.e8cq").encode()) == 0
    ref.q8c_read_close()
