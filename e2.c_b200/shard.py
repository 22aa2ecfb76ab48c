"""Batch sharding of an embedding job over GPUs: whole sequences per rank, weights replicated, one
gather of the pooled embeddings at the end.

The encoder has no interaction between sequences (e2.c src/text.c:842-886 loops sequences
independently inside a batch), so a job of many sequences splits into independent units:

  1. bucket: every sequence is padded to a multiple of `pad` tokens (its bucket length); sequences
     of one bucket run together as [batch][bucket_len] passes with a validity mask;
  2. assign: sequences go to ranks by longest-processing-time-first on the cost model
        cost(S) = layers * (macs_per_token * S + attn_macs * S^2)
     (int8 GEMM MACs grow with the tokens, attention with the square of the padded length), which
     keeps the ranks' finishing times within one sequence of each other;
  3. gather: each rank embeds its share in (bucket, position) order, the pooled rows are gathered
     to every rank (one collective, padded to the largest share), and the original order is
     restored from the gathered sequence indices.

Everything here is host logic (numpy + torch.distributed); the device work is the encoder's.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np

# int8 MACs per token and layer of the synthetic encoder (hidden 768, 3 + 1 heads of 256, FFN 1152):
# 768 * (768 + 256 + 256 + 768) + 3 * 768 * 1152
MACS_PER_TOKEN = 4_227_072
# attention MACs per (query, key) pair and layer: QK and PV over 3 heads of 256
ATTN_MACS = 2 * 3 * 256


def log_uniform_lengths(rng: np.random.Generator, n: int, lo: int = 32, hi: int = 2048) -> np.ndarray:
    """Sequence lengths floor(exp(U[ln lo, ln hi])) (benchmark config 4)."""
    return np.floor(np.exp(rng.uniform(np.log(lo), np.log(hi), size=n))).astype(np.int64).clip(lo, hi)


def bucket_length(lengths: np.ndarray, pad: int = 64) -> np.ndarray:
    """The padded length each sequence runs at: its length rounded up to a multiple of `pad`."""
    return ((np.asarray(lengths, np.int64) + pad - 1) // pad) * pad


def sequence_cost(padded: np.ndarray, layers: int = 24, macs_per_token: int = MACS_PER_TOKEN,
                  attn_macs: int = ATTN_MACS) -> np.ndarray:
    s = np.asarray(padded, np.float64)
    return layers * (macs_per_token * s + attn_macs * s * s)


def lpt_assign(costs: np.ndarray, world: int) -> list[np.ndarray]:
    """Longest-processing-time-first: sequences in decreasing cost, each to the least-loaded rank.
    Returns, per rank, the sequence indices it owns (ascending)."""
    costs = np.asarray(costs, np.float64)
    order = np.argsort(-costs, kind="stable")
    heap = [(0.0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(int(i))
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


@dataclass
class Pass:
    """One device pass: `seqs` (global sequence indices) at padded length `length`."""
    length: int
    seqs: np.ndarray


def plan_passes(indices: np.ndarray, padded: np.ndarray, max_tokens: int) -> list[Pass]:
    """Group a rank's sequences by bucket length into passes of at most max_tokens tokens."""
    passes: list[Pass] = []
    idx = np.asarray(indices, np.int64)
    lens = np.asarray(padded, np.int64)[idx]
    for length in np.unique(lens):
        members = idx[lens == length]
        per = max(1, max_tokens // int(length))
        for k in range(0, len(members), per):
            passes.append(Pass(int(length), members[k:k + per]))
    return passes


def pack_batch(ids_of, lengths: np.ndarray, p: Pass) -> tuple[np.ndarray, np.ndarray]:
    """ids [batch][length] int32 and valid [batch][length] uint8 for a pass; ids_of(i) gives the
    token ids of sequence i (length lengths[i]); padding positions get id 0 and valid 0."""
    b = len(p.seqs)
    ids = np.zeros((b, p.length), np.int32)
    valid = np.zeros((b, p.length), np.uint8)
    for r, i in enumerate(p.seqs):
        n = int(lengths[i])
        ids[r, :n] = ids_of(int(i))
        valid[r, :n] = 1
    return ids, valid


def gather_embeddings(dist, shares: list, local_emb, n_total: int, device=None):
    """All-gather every rank's embedding rows and return the [n_total][dim] matrix in original
    sequence order (on every rank). `shares` is lpt_assign's result, which every rank computes
    identically from the same job, so the row counts and the sequence index of every gathered row
    are known without exchanging them: the only collective is one all-gather of each rank's rows,
    padded to the largest share."""
    import torch

    rank, world = dist.get_rank(), dist.get_world_size()
    if len(shares) != world:
        raise ValueError(f"{len(shares)} shares for a world of {world}")
    dim = local_emb.shape[1]
    mine = len(shares[rank])
    if local_emb.shape[0] != mine:
        raise ValueError(f"rank {rank} holds {local_emb.shape[0]} rows for a share of {mine}")
    cmax = max(len(s) for s in shares)
    emb = torch.zeros((cmax, dim), dtype=local_emb.dtype, device=device)
    emb[:mine] = local_emb
    g_emb = torch.empty((world * cmax, dim), dtype=local_emb.dtype, device=device)
    dist.all_gather_into_tensor(g_emb, emb)
    src = np.concatenate([r * cmax + np.arange(len(s)) for r, s in enumerate(shares)]).astype(np.int64)
    dst = np.concatenate([np.asarray(s, np.int64) for s in shares])
    out = torch.empty((n_total, dim), dtype=local_emb.dtype, device=device)
    out[torch.as_tensor(dst, device=device)] = g_emb[torch.as_tensor(src, device=device)]
    return out
