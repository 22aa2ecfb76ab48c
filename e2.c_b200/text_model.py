"""e2.c's own text tower (EmbeddingGemma-2) as a seeded random-init checkpoint, and its description
for the device (e2cuda_text_create).

No checkpoint exists in this environment, so the tensors e2.c's loader reads (src/e2.c:294-420: the
names, the shapes it checks, bf16) are drawn here from a fixed seed and written as a
``model.safetensors`` e2.c itself can load. The same tensors, quantised by the loader's per-row
weight quantiser (src/int8.c:19-66; bf16 -> fp32 is exact), give the device description without
e2.c, so a user of the library (and ``bench.py``) builds the tower from the arrays alone.

Attention in this tower has scale 1.0 over RMS-normalised q and k (src/text.c:6-9), so with
random-init q_norm / k_norm gains near 1 the logits of a 256-dim head have a standard deviation
near 16 and the softmax is close to one-hot: a bf16 rounding of one logit then moves which key wins.
The checkpoint here is tempered instead: the q_norm and k_norm gains are drawn around ``qk_gain``
(0.25 by default), which puts the logits' standard deviation near 1 for head dim 256 (1.4 for 512).
"""
from __future__ import annotations

import ctypes as C
import json
import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .synthetic import PackedWeight, quantize_weight_rows

FULL_LAYERS = (5, 11, 17, 23)  # src/text.c:268


@dataclass
class TextConfig:
    """The text tower's fixed geometry (src/e2.c:294-301, src/text.c:470-481, src/model.h:13-17)."""

    n_layers: int = 24
    hidden: int = 512
    intermediate: int = 2048
    ple_dim: int = 512
    n_heads: int = 4
    vocab: int = 262144
    out_dim: int = 768
    eps: float = 1e-6
    rope_theta_full: float = 1000000.0
    rope_theta_sliding: float = 10000.0
    window: int = 512
    max_seq: int = 2048

    def full(self, l: int) -> bool:
        return l in FULL_LAYERS

    def head_dim(self, l: int) -> int:
        return 512 if self.full(l) else 256

    def n_kv(self, l: int) -> int:
        return 1 if self.full(l) else 2

    def q_dim(self, l: int) -> int:
        return self.n_heads * self.head_dim(l)

    def kv_dim(self, l: int) -> int:
        return self.n_kv(l) * self.head_dim(l)

    @property
    def embed_scale(self) -> float:
        return float(np.float32(math.sqrt(self.hidden)))

    @property
    def ple_scale(self) -> float:
        return float(np.float32(1.0) / np.float32(math.sqrt(self.hidden)))


LAYER_PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
              "mlp.up_proj", "mlp.down_proj", "ple_block.per_layer_input_gate", "ple_block.per_layer_projection")
LAYER_NORM = ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm",
              "ple_block.post_per_layer_input_norm")


def tensor_shapes(cfg: TextConfig) -> dict[str, tuple[int, ...]]:
    """Every tensor the loader reads for the text tower, with the shape it checks."""
    D, I, P, L = cfg.hidden, cfg.intermediate, cfg.ple_dim, cfg.n_layers
    s = {
        "language_model.embed_tokens.weight": (cfg.vocab, D),
        "language_model.ple.per_layer_model_projection.weight": (L * P, D),
        "language_model.embedding_projection.weight": (cfg.out_dim, D),
        "language_model.ple.per_layer_projection_norm.weight": (P,),
        "language_model.norm.weight": (D,),
    }
    for l in range(L):
        p = f"language_model.layers.{l}."
        qd, kvd, hd = cfg.q_dim(l), cfg.kv_dim(l), cfg.head_dim(l)
        for name, shape in zip(LAYER_PROJ, ((qd, D), (kvd, D), (kvd, D), (D, qd), (I, D), (I, D), (D, I), (P, D), (D, P))):
            s[p + name + ".weight"] = shape
        for name in LAYER_NORM:
            s[p + name + ".weight"] = (D,)
        s[p + "self_attn.q_norm.weight"] = (hd,)
        s[p + "self_attn.k_norm.weight"] = (hd,)
        s[p + "layer_scalar"] = (1,)
    return s


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even (finite inputs), as uint16 bit patterns."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def random_tensors(cfg: TextConfig | None = None, seed: int = 0xE2C0DE + 7, qk_gain: float = 0.25,
                   weight_std: float = 0.02, table_std: float = 0.04) -> dict[str, np.ndarray]:
    """bf16 bit patterns (uint16) for every tensor of tensor_shapes(cfg), from one seed.

    Projections N(0, weight_std); the token table N(0, table_std) (x = row * sqrt(512) then has an
    RMS near 0.9); norm gains 1 + N(0, 0.1); q_norm / k_norm gains qk_gain * (1 + N(0, 0.1)); layer
    scalars 1 on every fourth layer, else uniform in [0.5, 1)."""
    cfg = cfg or TextConfig()
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in tensor_shapes(cfg).items():
        if name.endswith("layer_scalar"):
            l = int(name.split(".")[2])
            v = np.array([1.0 if l % 4 == 0 else rng.uniform(0.5, 1.0)], np.float32)
        elif name.endswith("q_norm.weight") or name.endswith("k_norm.weight"):
            v = np.float32(qk_gain) * (np.float32(1.0) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1))
        elif len(shape) == 1:
            v = np.float32(1.0) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
        elif name == "language_model.embed_tokens.weight":
            v = rng.standard_normal(shape, dtype=np.float32)
            v *= np.float32(table_std)
        else:
            v = rng.standard_normal(shape, dtype=np.float32)
            v *= np.float32(weight_std)
        out[name] = f32_to_bf16(v).reshape(shape)
    return out


def write_safetensors(path, tensors: dict[str, np.ndarray]) -> None:
    """A safetensors file of bf16 tensors (8-byte header length, JSON header padded so the data
    starts 8-byte aligned, tensors back to back)."""
    header, off = {}, 0
    for name, a in tensors.items():
        n = a.size * 2
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + n]}
        off += n
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - (8 + len(h)) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for a in tensors.values():
            f.write(np.ascontiguousarray(a, np.uint16).tobytes())


def read_safetensors(path) -> dict[str, np.ndarray]:
    """bf16 tensors of a safetensors file, as uint16 arrays (memory-mapped)."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    hlen = int.from_bytes(bytes(raw[:8]), "little")
    header = json.loads(bytes(raw[8:8 + hlen]))
    base = 8 + hlen
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        if e["dtype"] not in ("BF16", "bfloat16"):
            raise ValueError(f"{name}: {e['dtype']} (only bf16 is read here)")
        b0, b1 = e["data_offsets"]
        out[name] = raw[base + b0:base + b1].view(np.uint16).reshape(e["shape"])
    return out


class TextLayer(C.Structure):
    """e2cuda_text_layer (include/e2cuda.h)."""

    _fields_ = [(k, C.c_void_p) for k in ("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj")] + \
               [(k, C.c_void_p) for k in ("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "ple_norm", "q_norm",
                                          "k_norm")] + \
               [("layer_scalar", C.c_float), ("head_dim", C.c_int), ("n_kv_heads", C.c_int), ("window", C.c_int),
                ("rope_theta", C.c_float)]


class TextDesc(C.Structure):
    """e2cuda_text_desc (include/e2cuda.h)."""

    _fields_ = [(k, C.c_int) for k in ("n_layers", "hidden", "intermediate", "ple_dim", "n_heads", "vocab", "out_dim",
                                       "max_seq", "ablk")] + \
               [("eps", C.c_float), ("embed_scale", C.c_float), ("ple_scale", C.c_float)] + \
               [(k, C.c_void_p) for k in ("embed_tokens", "ple_model_proj", "embed_proj", "ple_proj_norm", "final_norm",
                                          "layers")]


def _addr(a) -> int:
    return a.ctypes.data if isinstance(a, np.ndarray) else C.addressof(a)


class TextWeights:
    """The tower's arrays in the form the device description points at: every projection quantised
    per row and packed as e2.c's e2_q8w (activation block `ablk` for the block sums), norm vectors
    fp32, the token table bf16."""

    def __init__(self, tensors: dict[str, np.ndarray], cfg: TextConfig | None = None, ablk: int = 128):
        self.cfg = cfg = cfg or TextConfig()
        self.ablk = ablk
        self._keep = []
        shapes = tensor_shapes(cfg)
        for name, shape in shapes.items():
            if tuple(tensors[name].shape) != shape:
                raise ValueError(f"{name}: shape {tuple(tensors[name].shape)}, expected {shape}")

        def q8(name):
            q, s = quantize_weight_rows(bf16_to_f32(tensors[name]))
            pw = PackedWeight(q, s, ablk)
            st = _Q8W()
            pw.fill(st)
            self._keep += [pw, st]
            return st

        def f32(name):
            v = np.ascontiguousarray(bf16_to_f32(tensors[name]).reshape(-1))
            self._keep.append(v)
            return v

        self.table = np.ascontiguousarray(tensors["language_model.embed_tokens.weight"], np.uint16)
        self.ple_model = q8("language_model.ple.per_layer_model_projection.weight")
        self.embed_proj = q8("language_model.embedding_projection.weight")
        self.ple_norm = f32("language_model.ple.per_layer_projection_norm.weight")
        self.final_norm = f32("language_model.norm.weight")
        self.layers = (TextLayer * cfg.n_layers)()
        self.q8 = []  # per layer: the nine packed projections, in LAYER_PROJ order
        for l in range(cfg.n_layers):
            p = f"language_model.layers.{l}."
            ws = [q8(p + n + ".weight") for n in LAYER_PROJ]
            self.q8.append(ws)
            norms = [f32(p + n + ".weight") for n in LAYER_NORM]
            qn, kn = f32(p + "self_attn.q_norm.weight"), f32(p + "self_attn.k_norm.weight")
            y = self.layers[l]
            for k, st in zip(("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj"), ws):
                setattr(y, k, C.addressof(st))
            for k, v in zip(("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "ple_norm"), norms):
                setattr(y, k, v.ctypes.data)
            y.q_norm, y.k_norm = qn.ctypes.data, kn.ctypes.data
            y.layer_scalar = float(bf16_to_f32(tensors[p + "layer_scalar"])[0])
            y.head_dim, y.n_kv_heads = cfg.head_dim(l), cfg.n_kv(l)
            y.window = -1 if cfg.full(l) else cfg.window
            y.rope_theta = cfg.rope_theta_full if cfg.full(l) else cfg.rope_theta_sliding

    def desc(self) -> TextDesc:
        c = self.cfg
        d = TextDesc()
        d.n_layers, d.hidden, d.intermediate, d.ple_dim = c.n_layers, c.hidden, c.intermediate, c.ple_dim
        d.n_heads, d.vocab, d.out_dim, d.max_seq, d.ablk = c.n_heads, c.vocab, c.out_dim, c.max_seq, self.ablk
        d.eps, d.embed_scale, d.ple_scale = c.eps, c.embed_scale, c.ple_scale
        d.embed_tokens = self.table.ctypes.data
        d.ple_model_proj, d.embed_proj = C.addressof(self.ple_model), C.addressof(self.embed_proj)
        d.ple_proj_norm, d.final_norm = self.ple_norm.ctypes.data, self.final_norm.ctypes.data
        d.layers = C.addressof(self.layers)
        return d


def _Q8W():
    from . import Q8W

    return Q8W()


def token_ids(rng: np.random.Generator, B: int, S: int, vocab: int = 262144) -> np.ndarray:
    return rng.integers(2, vocab, size=(B, S), dtype=np.int32)


def save(path, cfg: TextConfig | None = None, **kw) -> Path:
    """Write random_tensors(cfg, **kw) as <path>/model.safetensors; returns the directory."""
    d = Path(path)
    d.mkdir(parents=True, exist_ok=True)
    write_safetensors(d / "model.safetensors", random_tensors(cfg, **kw))
    return d
