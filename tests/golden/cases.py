"""Seeded input generators shared by the golden-fixture script, the tests and
the bench.  Each generator returns plain NumPy arrays (bf16 data as float32
values that bf16 represents exactly) so the same inputs can be handed to the
reference NumPy oracles, the CPU oracle and the CUDA path.

Shapes follow the reference tests (tests/test_paged_attention_kernel.py) and
BASELINE.json config 1.  The reference draws its inputs from unseeded
mx.random.normal; here numpy.random.default_rng(seed) stands in.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def _bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.view(np.float32)


def cast(a: np.ndarray, dtype: str) -> np.ndarray:
    """Rounds to `dtype`; float16 stays np.float16, bfloat16 comes back as float32 values."""
    if dtype == "float32":
        return a.astype(np.float32)
    if dtype == "float16":
        return a.astype(np.float32).astype(np.float16)
    if dtype == "bfloat16":
        return _bf16_round(a.astype(np.float32))
    raise ValueError(dtype)


def ref_setup_data(seed: int = 0) -> dict:
    """TestPagedAttentionKernels.setup_data (test_paged_attention_kernel.py:138-188).

    q/k/v are float32 (mx.random.normal), caches float16.  The fixture draws 64
    tokens but builds 75 slots (`k[:75]` of a 64-row array), so only the first
    64 slots are written; that quirk is kept.
    """
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((2, 8, 64), dtype=np.float32)
    k = rng.standard_normal((64, 4, 64), dtype=np.float32)
    v = rng.standard_normal((64, 4, 64), dtype=np.float32)
    k_cache = np.zeros((20, 4, 64 // 8, 16, 8), dtype=np.float16)
    v_cache = np.zeros((20, 4, 64, 16), dtype=np.float16)
    context_lens = np.array([25, 50], dtype=np.int32)
    block_tables = np.array([[0, 1, -1, -1], [2, 3, 4, 5]], dtype=np.int32)
    slot_mapping = np.array([i for i in range(25)] + [2 * 16 + i for i in range(50)], dtype=np.int32)
    return dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, context_lens=context_lens,
                block_tables=block_tables, slot_mapping=slot_mapping, num_kv_heads=4, scale=1.0 / math.sqrt(64),
                block_size=16, max_seq_len=64)


def ref_various(head_dim: int, block_size: int, seed: int = 1) -> dict:
    """test_various_shapes (test_paged_attention_kernel.py:248-282)."""
    rng = np.random.default_rng(seed + 7 * head_dim + block_size)
    q = rng.standard_normal((1, 4, head_dim), dtype=np.float32)
    k = rng.standard_normal((16, 2, head_dim), dtype=np.float32)
    v = rng.standard_normal((16, 2, head_dim), dtype=np.float32)
    k_cache = np.zeros((4, 2, head_dim // 8, block_size, 8), dtype=np.float16)
    v_cache = np.zeros((4, 2, head_dim, block_size), dtype=np.float16)
    return dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, context_lens=np.array([16], dtype=np.int32),
                block_tables=np.array([[0, 1, -1, -1] if block_size == 8 else [0, -1, -1, -1]], dtype=np.int32),
                slot_mapping=np.arange(16, dtype=np.int32), num_kv_heads=2, scale=1.0 / math.sqrt(head_dim),
                block_size=block_size, max_seq_len=16)


def ref_legacy_2048(seed: int = 2) -> dict:
    """test_context_longer_than_legacy_2048_limit (test_paged_attention_kernel.py:284-330)."""
    rng = np.random.default_rng(seed)
    head_dim, block_size, seq_len = 32, 16, 2112
    q = rng.standard_normal((1, 2, head_dim), dtype=np.float32)
    k = rng.standard_normal((seq_len, 1, head_dim), dtype=np.float32)
    v = rng.standard_normal((seq_len, 1, head_dim), dtype=np.float32)
    nb = math.ceil(seq_len / block_size)
    return dict(q=q, k=k, v=v, k_cache=np.zeros((nb, 1, head_dim // 8, block_size, 8), dtype=np.float16),
                v_cache=np.zeros((nb, 1, head_dim, block_size), dtype=np.float16),
                block_tables=np.arange(nb, dtype=np.uint32).reshape(1, -1),
                context_lens=np.array([seq_len], dtype=np.uint32), slot_mapping=np.arange(seq_len, dtype=np.int32),
                num_kv_heads=1, scale=1.0 / math.sqrt(head_dim), block_size=block_size, max_seq_len=seq_len)


def paged_batch(seed: int, dtype: str, num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                block_size: int, context_lens, extra_blocks: int = 3, cache_dtype: str | None = None) -> dict:
    """A batch in the vLLM layout built the way BASELINE.json config 1 says:
    block tables are a seeded random permutation of the pool's blocks and the
    cache is filled through reshape_and_cache with slots
    table[t // bs] * bs + t % bs.  Returns the (not yet filled) caches and the
    K/V token rows plus slots to fill them with."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(context_lens, dtype=np.int64)
    blocks_per_seq = [(-(-int(c) // block_size)) for c in lens]
    num_blocks = int(sum(blocks_per_seq)) + extra_blocks
    max_blocks = max(max(blocks_per_seq), 1)
    perm = rng.permutation(num_blocks).astype(np.int32)
    tables = np.full((num_seqs, max_blocks), -1, dtype=np.int32)
    pos = 0
    for b, nb in enumerate(blocks_per_seq):
        tables[b, :nb] = perm[pos:pos + nb]
        pos += nb
    total = int(lens.sum())
    q = cast(rng.standard_normal((num_seqs, num_heads, head_dim), dtype=np.float32), dtype)
    k = cast(rng.standard_normal((total, num_kv_heads, head_dim), dtype=np.float32), dtype)
    v = cast(rng.standard_normal((total, num_kv_heads, head_dim), dtype=np.float32), dtype)
    slots = np.empty(total, dtype=np.int64)
    o = 0
    for b, c in enumerate(lens):
        t = np.arange(int(c))
        slots[o:o + c] = tables[b, t // block_size].astype(np.int64) * block_size + t % block_size
        o += int(c)
    cd = cache_dtype or dtype
    store = np.float16 if cd == "float16" else np.float32
    x = 16 // (2 if cd in ("float16", "bfloat16") else 4)
    k_cache = np.zeros((num_blocks, num_kv_heads, head_dim // x, block_size, x), dtype=store)
    v_cache = np.zeros((num_blocks, num_kv_heads, head_dim, block_size), dtype=store)
    return dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, context_lens=lens.astype(np.int32),
                block_tables=tables, slot_mapping=slots.astype(np.int32), num_kv_heads=num_kv_heads,
                scale=1.0 / math.sqrt(head_dim), block_size=block_size,
                max_seq_len=int(max_blocks * block_size), dtype=dtype)


def config1(seed: int = 11, dtype: str = "float16") -> dict:
    """fp16, batch 8, 32 q / 8 kv heads, head_dim 128,
    block_size 16, context lens uniform in [1, 1024], N(0,1) inputs, scale 1/sqrt(128)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 1025, size=8)
    return paged_batch(seed + 1, dtype, 8, 32, 8, 128, 16, lens)
