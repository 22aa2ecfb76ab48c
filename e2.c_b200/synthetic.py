"""Seeded synthetic inputs and random-init int8 models for the benchmark configs 0-4.

No dataset or checkpoint exists for these configs (the synthetic encoder of config 2 is not a model
the reference can load), so every config is generated here from a fixed seed with the shapes and
distributions the benchmark configs name. Weights are quantised exactly as the reference's model loader
does (e2.c src/int8.c:19-66, the per-row weight quantiser with its -ffast-math scale forms), and packed
into the reference's quad-interleaved e2_q8w layout, so the device path consumes what a q8cache would
hold.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

INV127 = np.float32(1.0) / np.float32(127.0)  # fl(1/127)


def quantize_weight_rows(w: np.ndarray):
    """Per-row symmetric int8 (e2.c src/int8.c:37-55): scale = amax * fl(1/127) (1 for a zero row),
    q = rint(w * fl(127/amax)) saturated to +-127. Returns (q int8 [N][K], scale fp32 [N])."""
    w = np.ascontiguousarray(w, np.float32)
    amax = np.max(np.abs(w), axis=1)
    pos = amax > 0
    safe = np.where(pos, amax, np.float32(1.0)).astype(np.float32)
    inv = np.where(pos, np.float32(127.0) / safe, np.float32(1.0)).astype(np.float32)
    scale = np.where(pos, (amax * INV127).astype(np.float32), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint((w * inv[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale


@dataclass
class PackedWeight:
    """A reference-layout e2_q8w (quad-interleaved) whose arrays live in numpy."""

    q: np.ndarray          # plain [N][K] int8 (kept for the oracle / device upload)
    scale: np.ndarray      # [N]
    ablk: int
    packed: np.ndarray = field(init=False)
    scale_pad: np.ndarray = field(init=False)
    bsq: np.ndarray = field(init=False)

    def __post_init__(self):
        N, K = self.q.shape
        npad, kq = (N + 7) // 8 * 8, (K + 3) // 4
        qp = np.zeros((npad, kq * 4), np.int8)
        qp[:N, :K] = self.q
        # [N/8][8][K/4][4] -> [N/8][K/4][8][4] (e2.c src/int8.h:14-18)
        self.packed = np.ascontiguousarray(qp.reshape(npad // 8, 8, kq, 4).transpose(0, 2, 1, 3)).reshape(-1)
        self.scale_pad = np.zeros(npad, np.float32)
        self.scale_pad[:N] = self.scale
        nb = (K + self.ablk - 1) // self.ablk
        sums = np.zeros((nb, npad), np.int32)
        for b in range(nb):
            sums[b, :N] = self.q[:, b * self.ablk:(b + 1) * self.ablk].astype(np.int32).sum(axis=1)
        self.bsq = np.ascontiguousarray(sums)

    @property
    def N(self) -> int:
        return self.q.shape[0]

    @property
    def K(self) -> int:
        return self.q.shape[1]

    def fill(self, s) -> None:
        """Point a ctypes e2_q8w-layout structure (Q8W) at these arrays."""
        s.w = self.packed.ctypes.data_as(C.POINTER(C.c_int8))
        s.bsq = self.bsq.ctypes.data_as(C.POINTER(C.c_int32))
        s.scale = self.scale_pad.ctypes.data_as(C.POINTER(C.c_float))
        s.N, s.K = self.N, self.K
        s.nblocks = self.bsq.shape[0]
        s.Npad = self.packed.size // (((self.K + 3) // 4) * 4)
        s.out_min, s.out_max = -1e31, 1e31
        s.borrowed = 1


def packed_weight(rng: np.random.Generator, N: int, K: int, std: float, ablk: int) -> PackedWeight:
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(std)).astype(np.float32)
    q, s = quantize_weight_rows(w)
    return PackedWeight(q, s, ablk)


# ------------------------------------------------------------------------------ config 0 / 3 data
OUTLIER_CHANNELS = (3, 97, 311, 600)


def activations(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    """N(0,1) activations with four fixed outlier channels x20 (config 0)."""
    x = rng.standard_normal((M, K), dtype=np.float32)
    for c in OUTLIER_CHANNELS:
        if c < K:
            x[:, c] *= np.float32(20.0)
    return x


# ------------------------------------------------------------------------------ config 2 model
@dataclass
class EncoderConfig:
    n_layers: int = 24
    hidden: int = 768
    n_heads: int = 3
    n_kv_heads: int = 1
    head_dim: int = 256
    ffn: int = 1152
    vocab: int = 262144
    dense_hidden: int = 3072
    out_dim: int = 768
    rope_theta: float = 10000.0
    eps: float = 1e-6
    attn_scale: float = 1.0 / 16.0      # 1/sqrt(head_dim); the config leaves the scale open
    embed_scale: float | None = None    # sqrt(hidden), as the reference's loader (e2.c src/e2.c:298)
    weight_std: float = 0.02
    norm_std: float = 0.1
    max_seq: int = 2048

    def __post_init__(self):
        if self.embed_scale is None:
            self.embed_scale = float(np.float32(math.sqrt(self.hidden)))


@dataclass
class EncoderWeights:
    cfg: EncoderConfig
    ablk: int
    table: np.ndarray
    table_scale: np.ndarray
    layers: list            # per layer dict: wq wk wv wo wg wu wd (PackedWeight) + norms
    final_norm: np.ndarray
    dense1: PackedWeight
    dense2: PackedWeight


def encoder_weights(cfg: EncoderConfig, seed: int = 0xE2C0DE + 2, ablk: int | None = None) -> EncoderWeights:
    rng = np.random.default_rng(seed)
    ablk = ablk or cfg.hidden
    D, GD, Dh, I = cfg.hidden, cfg.n_heads * cfg.head_dim, cfg.head_dim, cfg.ffn
    table_f = rng.standard_normal((cfg.vocab, D), dtype=np.float32)
    table, table_scale = quantize_weight_rows(table_f)
    del table_f

    def gamma(n):
        return (np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(cfg.norm_std)).astype(np.float32)

    s = cfg.weight_std
    layers = []
    for _ in range(cfg.n_layers):
        layers.append(dict(
            wq=packed_weight(rng, GD, D, s, ablk),
            wk=packed_weight(rng, cfg.n_kv_heads * Dh, D, s, ablk),
            wv=packed_weight(rng, cfg.n_kv_heads * Dh, D, s, ablk),
            wo=packed_weight(rng, D, GD, s, ablk if ablk != D else GD),
            wg=packed_weight(rng, I, D, s, ablk),
            wu=packed_weight(rng, I, D, s, ablk),
            wd=packed_weight(rng, D, I, s, ablk if ablk != D else I),
            input_ln=gamma(D), post_attn_ln=gamma(D), pre_ffn_ln=gamma(D), post_ffn_ln=gamma(D),
            q_norm=gamma(Dh), k_norm=gamma(Dh),
        ))
    final = gamma(D)
    dense1 = packed_weight(rng, cfg.dense_hidden, D, s, ablk)
    dense2 = packed_weight(rng, cfg.out_dim, cfg.dense_hidden, s, ablk if ablk != D else cfg.dense_hidden)
    return EncoderWeights(cfg, ablk, table, table_scale, layers, final, dense1, dense2)


def token_batch(rng: np.random.Generator, B: int, S: int, vocab: int) -> np.ndarray:
    """Token ids uniform in [2, vocab) (config 2)."""
    return rng.integers(2, vocab, size=(B, S), dtype=np.int32)


def log_uniform_lengths(rng: np.random.Generator, n: int, lo: int = 32, hi: int = 2048) -> np.ndarray:
    """Config-4 sequence lengths: floor(exp(U[ln lo, ln hi]))."""
    return np.floor(np.exp(rng.uniform(math.log(lo), math.log(hi), size=n))).astype(np.int32)


def fill_desc(w: EncoderWeights, q8w_type, desc_type, ptr_float_type=C.POINTER(C.c_float)):
    """Build an e2cuda_encoder_desc / e2o_encoder-compatible structure over `w`'s arrays. Returns
    (desc, keepalive) — keep the second object alive as long as the first is used."""
    cfg, L = w.cfg, w.cfg.n_layers
    keep = []

    def q8w_array(key):
        arr = (q8w_type * L)()
        for i, lay in enumerate(w.layers):
            lay[key].fill(arr[i])
        keep.append(arr)
        return arr

    def ptr_array(key):
        arr = (ptr_float_type * L)()
        for i, lay in enumerate(w.layers):
            arr[i] = lay[key].ctypes.data_as(ptr_float_type)
        keep.append(arr)
        return arr

    d = desc_type()
    for k in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "dense_hidden", "out_dim"):
        setattr(d, k, getattr(cfg, k))
    if hasattr(d, "max_seq"):
        d.max_seq = cfg.max_seq
        d.ablk = w.ablk
    d.rope_theta, d.eps, d.attn_scale, d.embed_scale = cfg.rope_theta, cfg.eps, cfg.attn_scale, cfg.embed_scale
    d.table = w.table.ctypes.data_as(C.POINTER(C.c_int8))
    d.table_scale = w.table_scale.ctypes.data_as(ptr_float_type)
    for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
        setattr(d, k, C.cast(q8w_array(k), type(getattr(d, k))))
    for k in ("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "q_norm", "k_norm"):
        setattr(d, k, C.cast(ptr_array(k), type(getattr(d, k))))
    d.final_norm = w.final_norm.ctypes.data_as(ptr_float_type)
    d1, d2 = q8w_type(), q8w_type()
    w.dense1.fill(d1)
    w.dense2.fill(d2)
    keep += [d1, d2]
    d.dense1 = C.pointer(d1)
    d.dense2 = C.pointer(d2)
    keep.append(w)
    return d, keep
