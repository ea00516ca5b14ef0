"""Multi-GPU layout of the paged-KV decode: one process per GPU, KV pool sharded
by KV head (tensor-parallel attention layout).

Decode attention is independent per KV head, so a rank that owns KV heads
[h0, h1) and their G query heads each computes its slice of the output with no
exchange; block tables and context lengths are replicated.  When there are
fewer KV heads than ranks (e.g. 4 KV heads on 8 GPUs), ranks are grouped per
KV head and the sequences are split between the ranks of a group, balanced by
token count.  No collective is needed for the attention itself; gathering the
per-head outputs onto one rank is the caller's choice (an NCCL all-gather of
[B, Hq/N, D] slices).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ShardPlan:
    """What one rank computes."""

    rank: int
    world_size: int
    kv_heads: tuple[int, int]   # [start, end) of the KV heads this rank owns
    q_heads: tuple[int, int]    # [start, end) of the matching query heads
    seqs: np.ndarray            # indices of the sequences this rank attends (all of them unless heads < ranks)

    @property
    def num_kv_heads(self) -> int:
        return self.kv_heads[1] - self.kv_heads[0]

    @property
    def num_q_heads(self) -> int:
        return self.q_heads[1] - self.q_heads[0]


def split_by_tokens(context_lens, parts: int) -> list[np.ndarray]:
    """Splits sequence indices into `parts` contiguous groups of near-equal total
    tokens (greedy on the prefix sum)."""
    lens = np.asarray(context_lens, dtype=np.int64)
    n = len(lens)
    if parts <= 1 or n == 0:
        return [np.arange(n)]
    csum = np.cumsum(lens)
    total = csum[-1] if n else 0
    cuts = [0]
    for k in range(1, parts):
        target = total * k / parts
        cut = int(np.searchsorted(csum, target, side="left")) + 1
        cut = min(max(cut, cuts[-1]), n)
        cuts.append(cut)
    cuts.append(n)
    return [np.arange(cuts[i], cuts[i + 1]) for i in range(parts)]


def plan(num_heads: int, num_kv_heads: int, world_size: int, rank: int, context_lens) -> ShardPlan:
    """Shard plan of `rank` for a decode over `context_lens`."""
    if num_kv_heads <= 0 or num_heads % num_kv_heads:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if not 0 <= rank < world_size:
        raise ValueError("rank out of range")
    G = num_heads // num_kv_heads
    n = len(context_lens)
    if num_kv_heads >= world_size:
        if num_kv_heads % world_size:
            raise ValueError(f"{num_kv_heads} kv heads do not shard evenly over {world_size} ranks")
        per = num_kv_heads // world_size
        kv = (rank * per, (rank + 1) * per)
        return ShardPlan(rank, world_size, kv, (kv[0] * G, kv[1] * G), np.arange(n))
    if world_size % num_kv_heads:
        raise ValueError(f"{world_size} ranks do not group evenly over {num_kv_heads} kv heads")
    group = world_size // num_kv_heads  # ranks per KV head
    h = rank // group
    part = rank % group
    seqs = split_by_tokens(context_lens, group)[part]
    return ShardPlan(rank, world_size, (h, h + 1), (h * G, (h + 1) * G), seqs)


def assemble(outputs: list[np.ndarray], plans: list[ShardPlan], num_seqs: int, num_heads: int) -> np.ndarray:
    """Reassembles per-rank outputs [len(seqs), q heads, D] into [B, Hq, D] (host-side check / gather)."""
    D = outputs[0].shape[-1]
    full = np.zeros((num_seqs, num_heads, D), dtype=outputs[0].dtype)
    for out, p in zip(outputs, plans):
        full[p.seqs, p.q_heads[0]:p.q_heads[1]] = out
    return full
