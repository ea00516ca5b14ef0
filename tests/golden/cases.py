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


# ---------------------------------------------------------------------------
# BASELINE.json workloads (configs 2-5) for the bench and the large parity tests.
# Only the host-side structure is built here (lengths, block tables, slots);
# K/V contents are drawn on the device by the caller.
# ---------------------------------------------------------------------------
BASELINE = {
    2: dict(name="llama3-8b-batched-decode", layers=32, batch=256, hq=32, hkv=8, d=128, bs=16, partition=0),
    3: dict(name="128k-batch1-splitk-decode", layers=1, batch=1, hq=64, hkv=8, d=128, bs=32, partition=512),
    4: dict(name="radix-shared-prefix-decode", layers=1, batch=64, hq=64, hkv=8, d=128, bs=16, partition=0,
            prefix=2048, tail=256, l2_flush=True),
    5: dict(name="mixed-continuous-batch-step", layers=1, batch=512, hq=28, hkv=4, d=128, bs=32, partition=0,
            prefill_chunks=16, chunk=512, lognormal_median=1500.0, lognormal_sigma=1.0, clip=(16, 32768)),
}


def _tables_from_free_list(n_blocks_per_seq, free_list):
    mb = max(max(n_blocks_per_seq), 1)
    tables = np.zeros((len(n_blocks_per_seq), mb), np.int32)
    o = 0
    for b, n in enumerate(n_blocks_per_seq):
        tables[b, :n] = free_list[o:o + n]
        tables[b, n:] = free_list[o] if n else 0  # padding, never read
        o += n
    return tables, o


def baseline_workload(config: int, batch: int | None = None) -> dict:
    """One decode step of BASELINE config `config`.

    Returns the sequences' context length before the step (`lens`), their block
    tables covering lens + 1 tokens, the slot each sequence's new token is
    appended to (`decode_slots`), the pool size, and for config 5 the slots of
    the step's prefill-chunk tokens.  `batch` shrinks the batch (profiling)."""
    cfg = dict(BASELINE[config])
    if batch:
        cfg["batch"] = batch
    B, bs = cfg["batch"], cfg["bs"]
    prefill_slots = np.zeros(0, np.int32)
    if config == 2:
        # seed 2121: the draw's mean (2304.4 tokens) is U[512, 4096]'s expectation, so tokens/s is not
        # flattered by a light draw (KV per layer 2.42 GB, as the uniform distribution implies)
        lens = np.random.default_rng(2121).integers(512, 4096 + 1, size=B).astype(np.int64)
        nblk = [(-(-int(c + 1) // bs)) for c in lens]
        free = np.random.default_rng(7).permutation(int(sum(nblk))).astype(np.int32)
        tables, used = _tables_from_free_list(nblk, free)
        num_blocks = used
    elif config == 3:
        lens = np.full(B, 131072 - 1, np.int64)
        nblk = [(-(-int(c + 1) // bs)) for c in lens]
        free = np.random.default_rng(8).permutation(int(sum(nblk))).astype(np.int32)
        tables, num_blocks = _tables_from_free_list(nblk, free)
    elif config == 4:
        pre_blocks = cfg["prefix"] // bs
        tail_blocks = cfg["tail"] // bs
        num_blocks = pre_blocks + B * tail_blocks
        free = np.random.default_rng(9).permutation(num_blocks).astype(np.int32)
        prefix = free[:pre_blocks]
        tables = np.zeros((B, pre_blocks + tail_blocks), np.int32)
        for b in range(B):
            tables[b, :pre_blocks] = prefix
            tables[b, pre_blocks:] = free[pre_blocks + b * tail_blocks: pre_blocks + (b + 1) * tail_blocks]
        lens = np.full(B, cfg["prefix"] + cfg["tail"] - 1, np.int64)
    elif config == 5:
        rng = np.random.default_rng(10)
        lo, hi = cfg["clip"]
        lens = np.clip(rng.lognormal(np.log(cfg["lognormal_median"]), cfg["lognormal_sigma"], B), lo, hi)
        lens = lens.astype(np.int64)
        nblk = [(-(-int(c + 1) // bs)) for c in lens]
        chunk_blocks = cfg["chunk"] // bs
        num_blocks = int(sum(nblk)) + cfg["prefill_chunks"] * chunk_blocks
        free = rng.permutation(num_blocks).astype(np.int32)  # seeded shuffled block free list
        tables, used = _tables_from_free_list(nblk, free)
        pre = free[used:used + cfg["prefill_chunks"] * chunk_blocks].astype(np.int64)
        t = np.arange(cfg["prefill_chunks"] * cfg["chunk"])
        prefill_slots = (pre[t // bs] * bs + t % bs).astype(np.int32)
    else:
        raise ValueError(config)
    decode_slots = (tables[np.arange(B), lens // bs].astype(np.int64) * bs + lens % bs).astype(np.int32)
    return dict(cfg=cfg, lens=lens, tables=tables, num_blocks=int(num_blocks), decode_slots=decode_slots,
                prefill_slots=prefill_slots, max_seq_len=int(tables.shape[1] * bs))


def unique_kv_bytes(tables, lens_after, hkv, d, bs, elem=2):
    """K+V bytes a decode must read when shared blocks are read once: every
    distinct block counts its largest used prefix of tokens once."""
    used = {}
    for b, c in enumerate(lens_after):
        nb = -(-int(c) // bs)
        for i in range(nb):
            blk = int(tables[b, i])
            toks = min(bs, int(c) - i * bs)
            if toks > used.get(blk, 0):
                used[blk] = toks
    return sum(used.values()) * hkv * d * elem * 2
