"""e2.c_b200 — Python mirror of the e2cuda C ABI (include/e2cuda.h).

The product is ``libe2cuda.so`` in this directory: sm_100a kernels plus a C11 host library. This
module binds it with ctypes so tests and ``bench.py`` call the same entry points an e2.c build would
bind. Device buffers are torch CUDA tensors, used only as memory and streams.

The directory name contains a dot, so import it by path::

    spec = importlib.util.spec_from_file_location("e2c_b200", "e2.c_b200/__init__.py")

There is no CPU fallback: every op raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libe2cuda.so"
HEADER = PKG.parent / "include" / "e2cuda.h"

f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int32)
u8p = C.POINTER(C.c_uint8)
vp = C.c_void_p


class E2CudaError(RuntimeError):
    pass


class Q8W(C.Structure):
    """e2cuda_q8w == the reference's e2_q8w (e2.c src/int8.h:79-92)."""

    _fields_ = [("w", i8p), ("bsq", i32p), ("scale", f32p), ("N", C.c_int), ("K", C.c_int),
                ("nblocks", C.c_int), ("Npad", C.c_int), ("out_min", C.c_float), ("out_max", C.c_float),
                ("borrowed", C.c_int)]


class W8(C.Structure):
    _fields_ = [("w", i8p), ("scale", f32p), ("N", C.c_int), ("K", C.c_int), ("rows", C.c_int), ("ld", C.c_int),
                ("out_min", C.c_float), ("out_max", C.c_float)]


class Epilogue(C.Structure):
    _fields_ = [("residual", f32p), ("ld_residual", C.c_int), ("dots", i32p)]


class EncoderDesc(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int), ("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
        ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("dense_hidden", C.c_int), ("out_dim", C.c_int),
        ("max_seq", C.c_int), ("ablk", C.c_int),
        ("rope_theta", C.c_float), ("eps", C.c_float), ("attn_scale", C.c_float), ("embed_scale", C.c_float),
        ("table", i8p), ("table_scale", f32p),
        ("wq", C.POINTER(Q8W)), ("wk", C.POINTER(Q8W)), ("wv", C.POINTER(Q8W)), ("wo", C.POINTER(Q8W)),
        ("wg", C.POINTER(Q8W)), ("wu", C.POINTER(Q8W)), ("wd", C.POINTER(Q8W)),
        ("input_ln", C.POINTER(f32p)), ("post_attn_ln", C.POINTER(f32p)), ("pre_ffn_ln", C.POINTER(f32p)),
        ("post_ffn_ln", C.POINTER(f32p)), ("q_norm", C.POINTER(f32p)), ("k_norm", C.POINTER(f32p)),
        ("final_norm", f32p), ("dense1", C.POINTER(Q8W)), ("dense2", C.POINTER(Q8W)),
    ]


class GemmArgs(C.Structure):
    """Mirror of e2c_gemm_args (csrc/launch.h), the launcher under e2cuda_i8_gemm: the fused
    epilogues (GELU-gate, per-head norm + RoPE, residual norm + quantise) are reached only through it. Used by the parity
    tests and by bench.py to time one encoder GEMM in isolation."""

    _fields_ = [("a", C.c_void_p), ("lda", C.c_int), ("a_scale", C.c_void_p), ("w", C.c_void_p), ("ldw", C.c_int),
                ("wrows", C.c_int), ("w_scale", C.c_void_p), ("M", C.c_int), ("K", C.c_int), ("ablk", C.c_int),
                ("n0", C.c_int), ("n1", C.c_int), ("epi", C.c_int), ("y", C.c_void_p), ("ldy", C.c_int),
                ("resid", C.c_void_p), ("ldr", C.c_int), ("dots", C.c_void_p), ("ldd", C.c_int),
                ("out_min", C.c_float), ("out_max", C.c_float), ("nq", C.c_int), ("q_out", C.c_void_p),
                ("k_out", C.c_void_p), ("vt_out", C.c_void_p), ("ldvt", C.c_int), ("seq_len", C.c_int),
                ("q_gamma", C.c_void_p), ("k_gamma", C.c_void_p), ("rope_cos", C.c_void_p),
                ("rope_sin", C.c_void_p), ("ldrope", C.c_int), ("eps", C.c_float), ("res", C.c_void_p), ("ldres", C.c_int),
                ("norm_g1", C.c_void_p), ("norm_g2", C.c_void_p), ("norm_gf", C.c_void_p), ("q8", C.c_void_p),
                ("ldq", C.c_int), ("q8_scale", C.c_void_p), ("status", C.c_void_p), ("ws", C.c_void_p),
                ("ws_bytes", C.c_size_t), ("norm_ls", C.c_float)]


EPI_F32, EPI_RESID, EPI_I32, EPI_GELU, EPI_QKV, EPI_NORMADD, EPI_GELUQ, EPI_QKVPB = 0, 1, 2, 3, 4, 5, 6, 7


def gemm_args(w: "Weight", qa, a_scales, M: int) -> GemmArgs:
    """Launcher arguments for weight `w` over per-token-quantised activations (all columns)."""
    a = GemmArgs()
    a.a, a.lda, a.a_scale = qa.data_ptr(), w.w8.ld, a_scales.data_ptr()
    a.w, a.ldw, a.wrows, a.w_scale = C.cast(w.w8.w, C.c_void_p), w.w8.ld, w.w8.rows, C.cast(w.w8.scale, C.c_void_p)
    a.M, a.K, a.ablk, a.n0, a.n1 = M, w.w8.ld, w.w8.ld, 0, w.N
    a.out_min, a.out_max = w.w8.out_min, w.w8.out_max
    return a


def gemm_raw(args: GemmArgs, stream=None) -> None:
    l = lib()
    _ok(0 if l.e2c_gemm(C.byref(args), _stream(stream)) == 0 else -1, "e2c_gemm: " + l.e2c_msg().decode())


# (name, restype, argtypes) of every entry point include/e2cuda.h declares
API = [
    ("e2cuda_last_error", C.c_char_p, []),
    ("e2cuda_device", C.c_char_p, []),
    ("e2cuda_check", C.c_int, [vp]),
    ("e2cuda_w8_from_q8w", C.c_int, [C.POINTER(Q8W), C.POINTER(W8)]),
    ("e2cuda_w8_from_int8", C.c_int, [i8p, f32p, C.c_int, C.c_int, C.POINTER(W8)]),
    ("e2cuda_w8_free", None, [C.POINTER(W8)]),
    ("e2cuda_quantize_rows", C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, vp]),
    ("e2cuda_i8_gemm", C.c_int, [C.POINTER(W8), vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Epilogue),
                                 vp, C.c_int, vp]),
    ("e2cuda_i8_linear_noalloc", C.c_int, [C.POINTER(W8), vp, C.c_int, C.c_int, vp, C.c_int, vp]),
    ("e2cuda_attention", C.c_int, [vp, vp, vp, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, vp]),
    ("e2cuda_attention_gqa", C.c_int, [vp, vp, vp, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_float, vp]),
    ("e2cuda_attention_window", C.c_int, [vp, vp, vp, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_float, C.c_int, vp]),
    ("e2cuda_ffn_create", vp, [C.POINTER(Q8W), C.POINTER(Q8W), C.POINTER(Q8W), f32p, C.c_float, C.c_int]),
    ("e2cuda_ffn_destroy", None, [vp]),
    ("e2cuda_ffn_forward", C.c_int, [vp, vp, C.c_int, vp, vp]),
    ("e2cuda_set_act_block", None, [C.c_int]),
    ("e2cuda_i8_quantize_host", None, [i8p, f32p, f32p, C.c_int, C.c_int, C.c_float, C.c_float]),
    ("e2cuda_i8_gemm_host", None, [f32p, i8p, f32p, C.POINTER(Q8W), C.c_int, C.c_int, C.c_int, C.c_int]),
    ("e2cuda_host_cache_clear", None, []),
    ("e2cuda_encoder_create", vp, [C.POINTER(EncoderDesc), C.c_int]),
    ("e2cuda_encoder_destroy", None, [vp]),
    ("e2cuda_encoder_embed_batch", C.c_int, [vp, i32p, u8p, C.c_int, C.c_int, f32p]),
    ("e2cuda_encoder_embed_batch_device", C.c_int, [vp, vp, vp, C.c_int, C.c_int, vp, vp]),
    ("e2cuda_encoder_stats", C.c_int, [vp, C.POINTER(C.c_long), C.POINTER(C.c_long), C.POINTER(C.c_double)]),
    ("e2cuda_q8c_open", vp, [C.c_char_p]),
    ("e2cuda_q8c_close", None, [vp]),
    ("e2cuda_q8c_version", C.c_int, [vp]),
    ("e2cuda_q8c_count", C.c_int, [vp]),
    ("e2cuda_q8c_entry", C.c_int, [vp, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                   C.POINTER(C.c_int64), C.POINTER(C.c_uint64)]),
    ("e2cuda_q8c_get", vp, [vp, C.c_char_p, C.c_int, C.POINTER(C.c_size_t)]),
    ("e2cuda_q8c_get_q8w", C.c_int, [vp, C.c_char_p, C.POINTER(Q8W)]),
    ("e2cuda_q8c_upload_w8", C.c_int, [vp, C.c_char_p, C.POINTER(W8)]),
    ("e2cuda_q8c_create", vp, [C.c_char_p]),
    ("e2cuda_q8c_put", C.c_int, [vp, C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_int64), vp, C.c_size_t]),
    ("e2cuda_q8c_put_q8w", C.c_int, [vp, C.c_char_p, C.POINTER(Q8W)]),
    ("e2cuda_q8c_put_w8", C.c_int, [vp, C.c_char_p, C.POINTER(Q8W)]),
    ("e2cuda_q8c_commit", C.c_int, [vp]),
    ("e2cuda_q8c_abort", None, [vp]),
    ("e2cuda_q8c_convert", C.c_int, [C.c_char_p, C.c_char_p]),
    ("e2cuda_text_create", vp, [vp, C.c_int]),
    ("e2cuda_text_destroy", None, [vp]),
    ("e2cuda_text_embed", C.c_int, [vp, i32p, C.c_int, f32p]),
    ("e2cuda_text_embed_batch", C.c_int, [vp, i32p, u8p, C.c_int, C.c_int, f32p]),
    ("e2cuda_text_embed_batch_device", C.c_int, [vp, vp, vp, C.c_int, C.c_int, vp, vp]),
    ("e2cuda_text_stats", C.c_int, [vp, C.POINTER(C.c_long), C.POINTER(C.c_long), C.POINTER(C.c_double)]),
]

Q8C_BF16, Q8C_F32, Q8C_Q8W, Q8C_W8 = 1, 2, 3, 4

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded libe2cuda.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise E2CudaError(f"{LIB_PATH} is missing: run __graft_entry__.build() (python e2.c_b200/build.py)")
        _lib = C.CDLL(str(LIB_PATH))
        for name, res, args in API:
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib.e2c_gemm.argtypes = [C.POINTER(GemmArgs), vp]
        _lib.e2c_gemm.restype = C.c_int
        _lib.e2c_msg.restype = C.c_char_p
    return _lib


def last_error() -> str:
    return (lib().e2cuda_last_error() or b"").decode()


def _ok(rc: int, what: str) -> None:
    if rc != 0:
        raise E2CudaError(f"{what}: {last_error()}")


def _torch():
    import torch

    if not torch.cuda.is_available():
        raise E2CudaError("no CUDA device: the e2cuda ops have no CPU path")
    return torch


def _ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def _stream(stream) -> int | None:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def check(stream=None) -> None:
    _ok(lib().e2cuda_check(_stream(stream)), "device check")


# ------------------------------------------------------------------------------------------ ops
def quantize_rows(x, ablk: int | None = None, lo: float = -math.inf, hi: float = math.inf, stream=None):
    """A1 on the device: x [M][K] fp32 -> (q [M][K] int8 signed, scales [M][K/ablk] fp32)."""
    torch = _torch()
    M, K = x.shape
    ablk = ablk or K
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, K // ablk), dtype=torch.float32, device=x.device)
    _ok(lib().e2cuda_quantize_rows(_ptr(x), _ptr(q), _ptr(s), M, K, ablk, lo, hi, _stream(stream)), "quantize_rows")
    return q, s


class Weight:
    """A device e2cuda_w8, from a reference-layout Q8W or from plain int8 rows + scales."""

    def __init__(self, *, q8w: Q8W | None = None, w: np.ndarray | None = None, scale: np.ndarray | None = None):
        self.w8 = W8()
        if q8w is not None:
            _ok(lib().e2cuda_w8_from_q8w(C.byref(q8w), C.byref(self.w8)), "w8_from_q8w")
        else:
            w = np.ascontiguousarray(w, np.int8)
            scale = np.ascontiguousarray(scale, np.float32)
            _ok(lib().e2cuda_w8_from_int8(w.ctypes.data_as(i8p), scale.ctypes.data_as(f32p), w.shape[0], w.shape[1],
                                         C.byref(self.w8)), "w8_from_int8")

    @property
    def N(self) -> int:
        return self.w8.N

    @property
    def K(self) -> int:
        return self.w8.K

    def free(self) -> None:
        if self.w8.w:
            lib().e2cuda_w8_free(C.byref(self.w8))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def i8_gemm(w: Weight, qa, a_scales, ablk: int | None = None, n0: int = 0, n1: int | None = None, residual=None,
            dots: bool = False, y=None, stream=None):
    """A3 on the device. Returns y [M][N] fp32 (columns outside [n0, n1) untouched), or with
    dots=True the raw int32 block dots [M][N][K/ablk]."""
    torch = _torch()
    M = qa.shape[0]
    ablk = ablk or w.K
    n1 = w.N if n1 is None else n1
    ep = Epilogue()
    if dots:
        out = torch.zeros((M, w.N, w.K // ablk), dtype=torch.int32, device=qa.device)
        ep.dots = C.cast(out.data_ptr(), i32p)
    else:
        out = y if y is not None else torch.zeros((M, w.N), dtype=torch.float32, device=qa.device)
        if residual is not None:
            ep.residual = C.cast(residual.data_ptr(), f32p)
            ep.ld_residual = residual.shape[1]
    _ok(lib().e2cuda_i8_gemm(C.byref(w.w8), _ptr(qa), _ptr(a_scales), M, ablk, n0, n1, C.byref(ep),
                             None if dots else _ptr(out), w.N, _stream(stream)), "i8_gemm")
    return out


# bytes of the fixed device array behind e2cuda_i8_linear_noalloc (E2CUDA_NOALLOC_SCRATCH_BYTES)
NOALLOC_SCRATCH_BYTES = 8 << 20


def i8_linear_noalloc(w: Weight, x, y, ablk: int | None = None, stream=None):
    """quantise(x) then the W8A8 GEMM into the caller's y [M][N] fp32, with no allocation in the
    library: the quantised activations live in the library's fixed per-device array. Returns y once
    written (the call synchronises `stream`)."""
    M = x.shape[0]
    ablk = ablk or w.K
    _ok(lib().e2cuda_i8_linear_noalloc(C.byref(w.w8), _ptr(x), M, ablk, _ptr(y), y.shape[1], _stream(stream)),
        "i8_linear_noalloc")
    return y


def attention(q, k, vt, valid, B: int, S: int, H: int, scale: float, stream=None):
    """A8 on the device: bf16 q [B*S][H*256], k [B*S][256], vt [B][256][ldvt] -> ctx fp32."""
    torch = _torch()
    ctx = torch.empty((B * S, H * 256), dtype=torch.float32, device=q.device)
    _ok(lib().e2cuda_attention(_ptr(q), _ptr(k), _ptr(vt), vt.shape[-1], _ptr(valid), _ptr(ctx), B, S, H, scale,
                               _stream(stream)), "attention")
    return ctx


def attention_gqa(q, k, vt, valid, B: int, S: int, H: int, KV: int, D: int, scale: float, stream=None):
    """bf16 attention with head dim D (64 or 256) and KV key/value heads: q [B*S][H*D], k [B*S][KV*D],
    vt [B][KV*D][ldvt] -> ctx fp32 [B*S][H*D]."""
    torch = _torch()
    ctx = torch.empty((B * S, H * D), dtype=torch.float32, device=q.device)
    _ok(lib().e2cuda_attention_gqa(_ptr(q), _ptr(k), _ptr(vt), vt.shape[-1], _ptr(valid), _ptr(ctx), B, S, H, KV, D,
                                   scale, _stream(stream)), "attention_gqa")
    return ctx


def attention_window(q, k, vt, valid, B: int, S: int, H: int, KV: int, D: int, scale: float, window: int = -1,
                     stream=None):
    """attention_gqa with a sliding window (|i - j| <= window; -1: none) and head dims 64, 256 or 512."""
    torch = _torch()
    ctx = torch.empty((B * S, H * D), dtype=torch.float32, device=q.device)
    _ok(lib().e2cuda_attention_window(_ptr(q), _ptr(k), _ptr(vt), vt.shape[-1], _ptr(valid), _ptr(ctx), B, S, H, KV, D,
                                      scale, window, _stream(stream)), "attention_window")
    return ctx


class FFN:
    """Config-1 fused FFN block on the device (e2cuda_ffn_*)."""

    def __init__(self, gate: Q8W, up: Q8W, down: Q8W, gamma: np.ndarray, eps: float, max_tokens: int):
        self._gamma = np.ascontiguousarray(gamma, np.float32)
        h = lib().e2cuda_ffn_create(C.byref(gate), C.byref(up), C.byref(down), self._gamma.ctypes.data_as(f32p),
                                    eps, max_tokens)
        if not h:
            raise E2CudaError(f"ffn_create: {last_error()}")
        self.h = h

    def forward(self, x, y=None, stream=None):
        torch = _torch()
        y = y if y is not None else torch.empty_like(x)
        _ok(lib().e2cuda_ffn_forward(self.h, _ptr(x), x.shape[0], _ptr(y), _stream(stream)), "ffn_forward")
        return y

    def __del__(self):
        try:
            if self.h:
                lib().e2cuda_ffn_destroy(self.h)
                self.h = None
        except Exception:
            pass


class Q8Cache:
    """A mapped .e8cq model cache (e2cuda_q8c_*): the reference's kinds 1-3 and kind 4, an int8
    weight in the device layout. Pointers it hands out live until close()."""

    def __init__(self, path):
        self.h = lib().e2cuda_q8c_open(str(path).encode())
        if not self.h:
            raise E2CudaError(f"q8c_open: {last_error()}")

    @property
    def version(self) -> int:
        return lib().e2cuda_q8c_version(self.h)

    def entries(self) -> list[tuple[str, int, tuple[int, ...], int]]:
        """(name, kind, dims, nbytes) of every index entry, in file order."""
        out = []
        for i in range(lib().e2cuda_q8c_count(self.h)):
            name, kind, ndim = C.c_char_p(), C.c_int(), C.c_int()
            dims, nb = (C.c_int64 * 4)(), C.c_uint64()
            _ok(lib().e2cuda_q8c_entry(self.h, i, C.byref(name), C.byref(kind), C.byref(ndim), dims, C.byref(nb)),
                "q8c_entry")
            out.append((name.value.decode(), kind.value, tuple(dims[:ndim.value]), nb.value))
        return out

    def blob(self, name: str, kind: int) -> np.ndarray:
        """The raw bytes stored under `name` (a copy)."""
        n = C.c_size_t()
        p = lib().e2cuda_q8c_get(self.h, name.encode(), kind, C.byref(n))
        if not p:
            raise E2CudaError(f"q8c_get: {last_error()}")
        return np.ctypeslib.as_array(C.cast(p, u8p), (n.value,)).copy() if n.value else np.zeros(0, np.uint8)

    def q8w(self, name: str) -> Q8W:
        q = Q8W()
        _ok(lib().e2cuda_q8c_get_q8w(self.h, name.encode(), C.byref(q)), "q8c_get_q8w")
        return q

    def upload_w8(self, name: str) -> "Weight":
        """A kind-4 entry copied to the device as is (a kind-3 one repacked on the way)."""
        wt = Weight.__new__(Weight)
        wt.w8 = W8()
        _ok(lib().e2cuda_q8c_upload_w8(self.h, name.encode(), C.byref(wt.w8)), "q8c_upload_w8")
        return wt

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().e2cuda_q8c_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Q8CacheWriter:
    """e2cuda_q8c_create / put / commit: a new .e8cq file, renamed into place by commit()."""

    def __init__(self, path):
        self.h = lib().e2cuda_q8c_create(str(path).encode())
        if not self.h:
            raise E2CudaError(f"q8c_create: {last_error()}")

    def put(self, name: str, kind: int, arr: np.ndarray) -> None:
        a = np.array(arr, order="C", copy=None)  # keeps rank 0 (np.ascontiguousarray would not)
        dims = (C.c_int64 * 4)(*a.shape)
        _ok(lib().e2cuda_q8c_put(self.h, name.encode(), kind, a.ndim, dims, a.ctypes.data_as(vp), a.nbytes), "q8c_put")

    def put_q8w(self, name: str, q) -> None:
        _ok(lib().e2cuda_q8c_put_q8w(self.h, name.encode(), C.cast(C.byref(q), C.POINTER(Q8W))), "q8c_put_q8w")

    def put_w8(self, name: str, q) -> None:
        _ok(lib().e2cuda_q8c_put_w8(self.h, name.encode(), C.cast(C.byref(q), C.POINTER(Q8W))), "q8c_put_w8")

    def commit(self) -> None:
        h, self.h = self.h, None
        _ok(lib().e2cuda_q8c_commit(h), "q8c_commit")

    def abort(self) -> None:
        if self.h:
            lib().e2cuda_q8c_abort(self.h)
            self.h = None

    def __del__(self):
        self.abort()


def q8c_convert(src, dst) -> None:
    """Rewrite cache `src` as `dst` with every kind-3 weight in kind 4 (the device layout)."""
    _ok(lib().e2cuda_q8c_convert(str(src).encode(), str(dst).encode()), "q8c_convert")


class Encoder:
    """The config-2 synthetic encoder (e2cuda_encoder_*). `weights` is a dict of host arrays / Q8W
    lists as produced by a synthetic-model builder; the library copies everything at create time."""

    def __init__(self, desc: EncoderDesc, keepalive, max_tokens: int):
        self._keep = keepalive
        self.desc = desc
        h = lib().e2cuda_encoder_create(C.byref(desc), max_tokens)
        if not h:
            raise E2CudaError(f"encoder_create: {last_error()}")
        self.h = h
        self.out_dim = desc.out_dim

    def embed_batch(self, ids: np.ndarray, valid: np.ndarray | None = None) -> np.ndarray:
        """Host buffers in and out (e2_hip_text_embed_batch's contract)."""
        ids = np.ascontiguousarray(ids, np.int32)
        B, S = ids.shape
        out = np.empty((B, self.out_dim), np.float32)
        v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
        _ok(lib().e2cuda_encoder_embed_batch(self.h, ids.ctypes.data_as(i32p), None if v is None else v.ctypes.data_as(u8p),
                                             B, S, out.ctypes.data_as(f32p)), "encoder_embed_batch")
        return out

    def embed_batch_into(self, ids, valid, out, host_ids=None) -> None:
        """Host pinned tensors (torch) in and out, without extra copies."""
        B, S = ids.shape
        _ok(lib().e2cuda_encoder_embed_batch(self.h, C.cast(ids.data_ptr(), i32p),
                                             None if valid is None else C.cast(valid.data_ptr(), u8p), B, S,
                                             C.cast(out.data_ptr(), f32p)), "encoder_embed_batch")

    def embed_batch_device(self, ids, valid, out, stream=None) -> None:
        B, S = ids.shape
        _ok(lib().e2cuda_encoder_embed_batch_device(self.h, _ptr(ids), _ptr(valid), B, S, _ptr(out), _stream(stream)),
            "encoder_embed_batch_device")

    def stats(self):
        calls, kern, ms = C.c_long(), C.c_long(), C.c_double()
        _ok(lib().e2cuda_encoder_stats(self.h, C.byref(calls), C.byref(kern), C.byref(ms)), "encoder_stats")
        return calls.value, kern.value, ms.value

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().e2cuda_encoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TextTower:
    """e2.c's own EmbeddingGemma-2 text tower on the device (e2cuda_text_*). `desc` is an
    e2cuda_text_desc (text_model.TextDesc, from text_model.TextWeights or filled by e2.c's loader);
    the library copies everything at create time."""

    def __init__(self, desc, max_tokens: int, keepalive=None):
        self._keep = keepalive
        h = lib().e2cuda_text_create(C.addressof(desc), max_tokens)
        if not h:
            raise E2CudaError(f"text_create: {last_error()}")
        self.h = h
        self.out_dim = desc.out_dim

    def embed_batch(self, ids: np.ndarray, valid: np.ndarray | None = None) -> np.ndarray:
        """Host buffers in and out (e2_hip_text_embed_batch's contract)."""
        ids = np.ascontiguousarray(ids, np.int32)
        B, S = ids.shape
        out = np.empty((B, self.out_dim), np.float32)
        v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
        _ok(lib().e2cuda_text_embed_batch(self.h, ids.ctypes.data_as(i32p), None if v is None else v.ctypes.data_as(u8p),
                                          B, S, out.ctypes.data_as(f32p)), "text_embed_batch")
        return out

    def embed(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        out = np.empty(self.out_dim, np.float32)
        _ok(lib().e2cuda_text_embed(self.h, ids.ctypes.data_as(i32p), ids.size, out.ctypes.data_as(f32p)), "text_embed")
        return out

    def embed_batch_into(self, ids, valid, out) -> None:
        """Host (pinned) torch tensors in and out, without extra copies."""
        B, S = ids.shape
        _ok(lib().e2cuda_text_embed_batch(self.h, C.cast(ids.data_ptr(), i32p),
                                          None if valid is None else C.cast(valid.data_ptr(), u8p), B, S,
                                          C.cast(out.data_ptr(), f32p)), "text_embed_batch")

    def embed_batch_device(self, ids, valid, out, stream=None) -> None:
        B, S = ids.shape
        _ok(lib().e2cuda_text_embed_batch_device(self.h, _ptr(ids), _ptr(valid), B, S, _ptr(out), _stream(stream)),
            "text_embed_batch_device")

    def stats(self):
        calls, kern, ms = C.c_long(), C.c_long(), C.c_double()
        _ok(lib().e2cuda_text_stats(self.h, C.byref(calls), C.byref(kern), C.byref(ms)), "text_stats")
        return calls.value, kern.value, ms.value

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().e2cuda_text_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
