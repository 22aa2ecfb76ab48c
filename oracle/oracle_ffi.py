"""ctypes access to the CPU checker. TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm import this
module. It wraps two kinds of library built by ``oracle/Makefile``:

* ``oracle/liboracle.so`` -- the plain-C restatement of the reference kernels (the "port");
* ``oracle/_ref/libe2ref_b<B>.so`` -- the reference's own kernel sources compiled with their own
  flags and ``-DE2_I8_BLOCK=<B>`` (absent where the reference sources were not available to build);
* ``oracle/_ref/libe2ref_text.so`` -- the reference's whole engine (loader + text tower), the
  checker of the device text tower (``RefText``).

Arrays are numpy; every wrapper checks dtype/contiguity and returns fresh outputs.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
PORT_LIB = HERE / "liboracle.so"

f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int32)
u8p = C.POINTER(C.c_uint8)


class Q8W(C.Structure):
    """Byte-for-byte the reference's e2_q8w (src/int8.h:79-92)."""

    _fields_ = [
        ("w", i8p),
        ("bsq", i32p),
        ("scale", f32p),
        ("N", C.c_int),
        ("K", C.c_int),
        ("nblocks", C.c_int),
        ("Npad", C.c_int),
        ("out_min", C.c_float),
        ("out_max", C.c_float),
        ("borrowed", C.c_int),
    ]

    def packed(self) -> np.ndarray:
        kq = (self.K + 3) // 4
        n = (self.Npad // 8) * kq * 32
        return np.ctypeslib.as_array(self.w, shape=(n,)).copy()

    def scales(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.scale, shape=(self.Npad,)).copy()

    def bsums(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.bsq, shape=(self.nblocks, self.Npad)).copy()


def _ptr(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data_as(t)


def _declare(lib: C.CDLL, with_ref: bool) -> C.CDLL:
    lib.e2o_quantize_blocks.argtypes = [i8p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float]
    lib.e2o_quantize_rows_signed.argtypes = [i8p, f32p, f32p, C.c_int, C.c_int, C.c_int]
    lib.e2o_q8w_from_f32.argtypes = [C.POINTER(Q8W), f32p, C.c_int, C.c_int, C.c_int]
    lib.e2o_q8w_free.argtypes = [C.POINTER(Q8W)]
    lib.e2o_q8w_unpack.argtypes = [C.POINTER(Q8W), i8p]
    lib.e2o_i8_gemm.argtypes = [f32p, i8p, f32p, C.POINTER(Q8W), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    lib.e2o_i8_gemm_plain.argtypes = [f32p, i32p, i8p, f32p, i8p, f32p, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_float, C.c_float]
    lib.e2o_rmsnorm.argtypes = [f32p, C.c_int, C.c_int, f32p, C.c_float]
    lib.e2o_norm_split.argtypes = [f32p, f32p, C.c_int, C.c_int, f32p, C.c_float]
    lib.e2o_norm_add.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, f32p, C.c_float]
    lib.e2o_gelu_tanh.argtypes = [f32p, C.c_size_t]
    lib.e2o_softmax.argtypes = [f32p, C.c_int]
    lib.e2o_rope_tables.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_float]
    lib.e2o_rope_rows.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32p, f32p]
    lib.e2o_fill_normal.argtypes = [f32p, C.c_size_t, C.c_uint64, C.c_float, C.c_float]
    lib.e2o_port_kernels.argtypes = [C.c_int]
    lib.e2o_port_kernels.restype = C.c_void_p
    lib.e2o_ffn_block.argtypes = [C.c_void_p, f32p, C.c_int, C.c_int, C.c_int, f32p, C.c_float,
                                  C.POINTER(Q8W), C.POINTER(Q8W), C.POINTER(Q8W), f32p, i8p, f32p,
                                  i8p, f32p, f32p]
    lib.e2o_encoder_forward.argtypes = [C.c_void_p, C.c_void_p, i32p, u8p, C.c_int, C.c_int, f32p,
                                        f32p, f32p]
    lib.e2o_attention_f32.argtypes = [C.c_void_p, f32p, f32p, f32p, f32p, u8p, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_float]
    if with_ref:
        lib.e2ref_block.restype = C.c_int
        lib.e2ref_init.argtypes = [C.c_int]
        lib.e2ref_init.restype = C.c_int
        lib.e2ref_backend.restype = C.c_char_p
        lib.e2ref_kernels.restype = C.c_void_p
        lib.e2ref_linear.argtypes = [f32p, C.c_int, C.c_int, C.POINTER(Q8W), i8p, f32p, f32p]
        qsig = [i8p, f32p, f32p, C.c_int, C.c_int, C.c_float, C.c_float]
        gsig = [f32p, i8p, f32p, C.POINTER(Q8W), C.c_int, C.c_int, C.c_int, C.c_int]
        for name in ("e2_quantize_blocks_avx512", "e2_quantize_blocks_scalar",
                     "e2_quantize_blocks_avx2", "e2_quantize_blocks_vnni"):
            getattr(lib, name).argtypes = qsig
        for name in ("e2_i8_gemm_avx512", "e2_i8_gemm_scalar", "e2_i8_gemm_avx2"):
            getattr(lib, name).argtypes = gsig
        lib.e2_q8w_from_f32.argtypes = [C.POINTER(Q8W), f32p, C.c_int, C.c_int]
        lib.e2_q8w_free.argtypes = [C.POINTER(Q8W)]
        lib.e2_cpu_init.argtypes = []
        lib.e2_meanpool_f32.argtypes = [f32p, f32p, C.c_int, C.c_int, u8p]
        lib.e2_l2norm_f32.argtypes = [f32p, C.c_int]
        lib.e2_sgemm_nn_range_avx512.argtypes = [f32p, C.c_int, f32p, C.c_int, f32p, C.c_int, C.c_int,
                                                 C.c_int, C.c_int, C.c_int, C.c_int]
    return lib


class Encoder(C.Structure):
    """e2o_encoder (e2_oracle.h): the config-2 synthetic encoder over packed e2_q8w weights."""

    _fields_ = [
        ("n_layers", C.c_int), ("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
        ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("dense_hidden", C.c_int), ("out_dim", C.c_int),
        ("rope_theta", C.c_float), ("eps", C.c_float), ("attn_scale", C.c_float), ("embed_scale", C.c_float),
        ("table", i8p), ("table_scale", f32p),
        ("wq", C.POINTER(Q8W)), ("wk", C.POINTER(Q8W)), ("wv", C.POINTER(Q8W)), ("wo", C.POINTER(Q8W)),
        ("wg", C.POINTER(Q8W)), ("wu", C.POINTER(Q8W)), ("wd", C.POINTER(Q8W)),
        ("input_ln", C.POINTER(f32p)), ("post_attn_ln", C.POINTER(f32p)), ("pre_ffn_ln", C.POINTER(f32p)),
        ("post_ffn_ln", C.POINTER(f32p)), ("q_norm", C.POINTER(f32p)), ("k_norm", C.POINTER(f32p)),
        ("final_norm", f32p), ("dense1", C.POINTER(Q8W)), ("dense2", C.POINTER(Q8W)),
    ]


_port = None
_refs: dict[int, C.CDLL | None] = {}
_mux = None


def port() -> C.CDLL:
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            raise FileNotFoundError(f"{PORT_LIB} missing: run make -C oracle (or __graft_entry__.build())")
        _port = _declare(C.CDLL(str(PORT_LIB)), False)
    return _port


_q8c: list = []


def ref_q8cache() -> C.CDLL | None:
    """The reference's .e8cq writer and reader (src/q8cache.c, built by oracle/Makefile), or None
    when the reference was not built here. Its state is global: one file open at a time."""
    if not _q8c:
        p = REF_DIR / "libe2ref_q8c.so"
        lib = None
        if p.exists():
            lib = C.CDLL(str(p))
            i64p = C.POINTER(C.c_int64)
            for name, res, args in [
                ("q8c_write_open", C.c_int, [C.c_char_p]),
                ("q8c_defer", C.c_int, [C.c_char_p, C.c_int, C.c_int, i64p, C.c_void_p, C.c_size_t]),
                ("q8c_put_q8w", C.c_int, [C.c_char_p, C.POINTER(Q8W)]),
                ("q8c_write_close", C.c_int, []),
                ("q8c_write_abort", None, []),
                ("q8c_read_open", C.c_int, [C.c_char_p]),
                ("q8c_read_close", None, []),
                ("q8c_get", C.c_void_p, [C.c_char_p, C.c_int, C.c_int, i64p, C.POINTER(C.c_size_t)]),
                ("q8c_get_q8w", C.c_int, [C.c_char_p, C.POINTER(Q8W)]),
                ("q8c_kind_of", C.c_int, [C.c_char_p]),
                ("q8c_error", C.c_char_p, []),
            ]:
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
        _q8c.append(lib)
    return _q8c[0]


def ref_available(block: int) -> bool:
    return (REF_DIR / f"libe2ref_b{block}.so").exists()


def ref(block: int, nthreads: int = 0) -> C.CDLL | None:
    """The reference build for activation block `block`, initialised with its pool; None if absent."""
    if block not in _refs:
        p = REF_DIR / f"libe2ref_b{block}.so"
        if not p.exists():
            _refs[block] = None
        else:
            lib = _declare(C.CDLL(str(p), mode=os.RTLD_LOCAL), True)
            if lib.e2ref_init(nthreads) < 0:
                raise RuntimeError("reference pool init failed")
            _refs[block] = lib
    return _refs[block]


def mux(nthreads: int = 0) -> C.CDLL | None:
    """oracle/_ref/libe2ref_mux.so: the reference kernels of every per-block build behind one table
    (per-row mode routes each call to the build with E2_I8_BLOCK = K). None if not built."""
    global _mux
    if _mux is None:
        p = REF_DIR / "libe2ref_mux.so"
        if not p.exists():
            return None
        lib = _declare(C.CDLL(str(p), mode=os.RTLD_LOCAL), False)
        lib.e2refmux_init.argtypes = [C.c_char_p, C.c_int]
        lib.e2refmux_init.restype = C.c_int
        lib.e2refmux_kernels.argtypes = [C.c_int]
        lib.e2refmux_kernels.restype = C.c_void_p
        lib.e2refmux_error.restype = C.c_char_p
        if lib.e2refmux_init(str(REF_DIR).encode(), nthreads) < 0:
            raise RuntimeError(lib.e2refmux_error().decode())
        _mux = lib
    return _mux


def kernels(which: str, ablk: int, nthreads: int = 0):
    """(library, kernel-table pointer) for which = "port" or "reference"; ablk 0 = per-row."""
    if which == "port":
        lib = port()
        return lib, lib.e2o_port_kernels(ablk)
    lib = mux(nthreads)
    if lib is None:
        raise FileNotFoundError("reference builds missing (oracle/_ref)")
    return lib, lib.e2refmux_kernels(ablk)


def ffn_block(which: str, x: np.ndarray, gamma: np.ndarray, eps: float, wg, wu, wd, ablk: int = 0,
              nthreads: int = 0, stages: bool = False):
    """Config-1 FFN block on the CPU (e2o_ffn_block). wg/wu/wd: synthetic.PackedWeight. Returns y, or
    (y, dict of stage dumps) with stages=True."""
    lib, k = kernels(which, ablk, nthreads)
    x = np.ascontiguousarray(x, np.float32)
    M, D = x.shape
    I = wg.N
    y = np.empty((M, D), np.float32)
    qs = [Q8W(), Q8W(), Q8W()]
    for q, w in zip(qs, (wg, wu, wd)):
        w.fill(q)
    nbD = 1 if ablk == 0 else D // ablk
    nbI = 1 if ablk == 0 else I // ablk
    xq = np.empty((M, D), np.int8) if stages else None
    xs = np.empty((M, nbD), np.float32) if stages else None
    hq = np.empty((M, I), np.int8) if stages else None
    hs = np.empty((M, nbI), np.float32) if stages else None
    gu = np.empty((M, 2 * I), np.float32) if stages else None
    g = np.ascontiguousarray(gamma, np.float32)
    rc = lib.e2o_ffn_block(k, _ptr(x, f32p), M, D, I, _ptr(g, f32p), eps, C.byref(qs[0]), C.byref(qs[1]),
                           C.byref(qs[2]), _ptr(y, f32p), _ptr(xq, i8p) if stages else None,
                           _ptr(xs, f32p) if stages else None, _ptr(hq, i8p) if stages else None,
                           _ptr(hs, f32p) if stages else None, _ptr(gu, f32p) if stages else None)
    if rc:
        raise RuntimeError("e2o_ffn_block failed")
    if not stages:
        return y
    return y, dict(xq=xq.view(np.uint8), xs=xs, hq=hq.view(np.uint8), hs=hs, gu=gu)


def encoder_forward(which: str, weights, ids: np.ndarray, valid: np.ndarray | None = None, nthreads: int = 0,
                    want_hidden: bool = False):
    """Config-2 encoder on the CPU (e2o_encoder_forward) over synthetic.EncoderWeights."""
    import importlib.util
    import sys

    syn = sys.modules.get("e2c_b200.synthetic")
    if syn is None:
        spec = importlib.util.spec_from_file_location("e2c_b200.synthetic", HERE.parent / "e2.c_b200" / "synthetic.py")
        syn = importlib.util.module_from_spec(spec)
        sys.modules["e2c_b200.synthetic"] = syn
        spec.loader.exec_module(syn)
    lib, k = kernels(which, 0 if weights.ablk == weights.cfg.hidden else weights.ablk, nthreads)
    desc, keep = syn.fill_desc(weights, Q8W, Encoder)
    ids = np.ascontiguousarray(ids, np.int32)
    B, S = ids.shape
    out = np.empty((B, weights.cfg.out_dim), np.float32)
    v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
    hid = np.empty((B * S, weights.cfg.hidden), np.float32) if want_hidden else None
    rc = lib.e2o_encoder_forward(k, C.addressof(desc), _ptr(ids, i32p), None if v is None else _ptr(v, u8p), B, S,
                                 _ptr(out, f32p), _ptr(hid, f32p) if want_hidden else None, None)
    del keep
    if rc:
        raise RuntimeError("e2o_encoder_forward failed")
    return (out, hid) if want_hidden else out


# ---------------------------------------------------------------------------------- numpy helpers
def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    port().e2o_fill_normal(_ptr(out, f32p), n, seed, mean, std)
    return out


def quantize_biased(x: np.ndarray, ablk: int, lo=-np.inf, hi=np.inf, lib=None, fn="e2o"):
    """(bytes q+128 as uint8 [M][K], scales [M][K/ablk]) from the port or a reference function."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    nb = (K + ablk - 1) // ablk
    q = np.empty((M, K), np.int8)
    s = np.empty((M, nb), np.float32)
    if lib is None:
        port().e2o_quantize_blocks(_ptr(q, i8p), _ptr(s, f32p), _ptr(x, f32p), M, K, ablk, lo, hi)
    else:
        getattr(lib, fn)(_ptr(q, i8p), _ptr(s, f32p), _ptr(x, f32p), M, K, lo, hi)
    return q.view(np.uint8), s


def quantize_signed(x: np.ndarray, ablk: int):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty((M, (K + ablk - 1) // ablk), np.float32)
    port().e2o_quantize_rows_signed(_ptr(q, i8p), _ptr(s, f32p), _ptr(x, f32p), M, K, ablk)
    return q, s


class Weight:
    """An e2_q8w built by the port or by the reference, freed with the matching library."""

    def __init__(self, w: np.ndarray, ablk: int, lib=None):
        w = np.ascontiguousarray(w, np.float32)
        self.N, self.K = w.shape
        self.q = Q8W()
        self._lib = lib
        if lib is None:
            rc = port().e2o_q8w_from_f32(C.byref(self.q), _ptr(w, f32p), self.N, self.K, ablk)
        else:
            rc = lib.e2_q8w_from_f32(C.byref(self.q), _ptr(w, f32p), self.N, self.K)
        if rc:
            raise MemoryError("q8w_from_f32 failed")

    def plain(self) -> np.ndarray:
        out = np.empty((self.N, self.K), np.int8)
        port().e2o_q8w_unpack(C.byref(self.q), _ptr(out, i8p))
        return out

    def scales(self) -> np.ndarray:
        return self.q.scales()[: self.N]

    def __del__(self):
        try:
            if self._lib is None:
                port().e2o_q8w_free(C.byref(self.q))
            else:
                self._lib.e2_q8w_free(C.byref(self.q))
        except Exception:
            pass


def gemm_plain(qa_signed: np.ndarray, as_: np.ndarray, w_plain: np.ndarray, ws: np.ndarray, ablk: int,
               want_dots: bool = False, out_min=-1e31, out_max=1e31):
    M, K = qa_signed.shape
    N = w_plain.shape[0]
    nb = (K + ablk - 1) // ablk
    y = np.empty((M, N), np.float32)
    dots = np.empty((M, N, nb), np.int32) if want_dots else None
    port().e2o_i8_gemm_plain(_ptr(y, f32p), _ptr(dots, i32p) if want_dots else None,
                             _ptr(np.ascontiguousarray(qa_signed), i8p),
                             _ptr(np.ascontiguousarray(as_, np.float32), f32p),
                             _ptr(np.ascontiguousarray(w_plain), i8p),
                             _ptr(np.ascontiguousarray(ws, np.float32), f32p), M, N, K, ablk,
                             out_min, out_max)
    return (y, dots) if want_dots else y


def gemm_ref(lib, qa_biased: np.ndarray, as_: np.ndarray, w: Weight, fn="e2_i8_gemm_avx512"):
    M, K = qa_biased.shape
    y = np.empty((M, w.N), np.float32)
    getattr(lib, fn)(_ptr(y, f32p), _ptr(np.ascontiguousarray(qa_biased).view(np.int8), i8p),
                     _ptr(np.ascontiguousarray(as_, np.float32), f32p), C.byref(w.q), M, w.N, 0, w.N)
    return y


# ------------------------------------------------------------------------------ e2.c's own text tower
REF_TEXT_LIB = REF_DIR / "libe2ref_text.so"
ATTN_TABLE, ATTN_F32, ATTN_I8 = -1, 0, 2  # e2_attn_kind (src/dispatch.h:26), -1: the dispatch table


class RefText:
    """e2.c's loader and text tower (oracle/ref_text.c over the reference's sources). One model per
    process (e2.c's own rule): `load` once, `embed_batch` any number of times."""

    def __init__(self):
        if not REF_TEXT_LIB.exists():
            raise FileNotFoundError(f"{REF_TEXT_LIB} was not built (make -C oracle needs the reference sources)")
        lib = C.CDLL(str(REF_TEXT_LIB))
        lib.ref_text_load.argtypes = [C.c_char_p, C.c_char_p]
        lib.ref_text_error.restype = C.c_char_p
        lib.ref_text_embed_batch.argtypes = [i32p, u8p, C.c_int, C.c_int, f32p]
        lib.ref_text_attention.argtypes = [C.c_int]
        lib.ref_text_describe.argtypes = [C.c_void_p, C.c_void_p]
        lib.ref_text_cuda_create.restype = C.c_void_p
        lib.e2_cuda_text_embed_batch.argtypes = [C.c_void_p, i32p, u8p, C.c_int, C.c_int, f32p]
        lib.e2_cuda_destroy.argtypes = [C.c_void_p]
        self.lib = lib

    def load(self, model_dir, cache_path) -> None:
        if self.lib.ref_text_load(str(model_dir).encode(), str(cache_path).encode()) != 0:
            raise RuntimeError(f"e2_load: {self.lib.ref_text_error().decode()}")

    def threads(self) -> int:
        return self.lib.ref_text_threads()

    def embed_batch(self, ids: np.ndarray, valid: np.ndarray | None = None, attention: int = ATTN_TABLE) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        B, S = ids.shape
        v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
        out = np.zeros((B, 768), np.float32)
        self.lib.ref_text_attention(attention)
        try:
            rc = self.lib.ref_text_embed_batch(_ptr(ids, i32p), None if v is None else _ptr(v, u8p), B, S, _ptr(out, f32p))
        finally:
            self.lib.ref_text_attention(ATTN_TABLE)
        if rc != 0:
            raise RuntimeError(f"e2_text_embed_batch: {self.lib.ref_text_error().decode()}")
        return out

    def describe(self, desc, layers) -> None:
        """Fill an e2cuda_text_desc (and its layer array) from the loaded e2_model: what the
        binding e2_cuda_create hands the library."""
        if self.lib.ref_text_describe(C.addressof(desc), C.addressof(layers)) != 0:
            raise RuntimeError("e2_cuda_describe: no int8 model loaded")

    def cuda_embed_batch(self, ids: np.ndarray, valid: np.ndarray | None = None) -> np.ndarray:
        """Through the binding as e2.c would call it: e2_cuda_create(m), e2_cuda_text_embed_batch."""
        g = self.lib.ref_text_cuda_create()
        if not g:
            raise RuntimeError("e2_cuda_create failed")
        try:
            ids = np.ascontiguousarray(ids, np.int32)
            B, S = ids.shape
            v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
            out = np.zeros((B, 768), np.float32)
            if self.lib.e2_cuda_text_embed_batch(g, _ptr(ids, i32p), None if v is None else _ptr(v, u8p), B, S,
                                                 _ptr(out, f32p)) != 0:
                raise RuntimeError("e2_cuda_text_embed_batch failed")
            return out
        finally:
            self.lib.e2_cuda_destroy(g)

    def free(self) -> None:
        self.lib.ref_text_free()
