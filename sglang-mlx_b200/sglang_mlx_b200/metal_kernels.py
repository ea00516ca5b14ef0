"""Kernel API of the B200 paged-KV path, signature-compatible with
sglang_mlx/metal_kernels.py (paged_attention_v1, reshape_and_cache,
copy_blocks, swap_blocks) plus the functions that file does not re-export
(reshape_and_cache_flash) or that sglang-mlx leaves unbuilt (the split-K decode
paged_attention_v2 and the auto-selecting paged_attention).

Arrays are DeviceArray objects or any DLPack CUDA array (a CUDA torch tensor,
CuPy, ...).  NumPy inputs are uploaded first, for convenience only.  Every
call goes through libkvcache.so; argument errors raise ValueError with the
reference's messages.  Work is queued on `stream` (default: the legacy default
stream) and is asynchronous like an unevaluated mx.array; `to_numpy()` or
`synchronize()` waits for it.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _lib, dtypes
from .device_array import DeviceArray, HostBuffer, _stream, asarray
from .dlpack import DLTensor, as_dltensor, describe

_L = _lib.lib

DEFAULT_PARTITION_SIZE = 512


def _dev(obj):
    """Arguments may be device arrays of any DLPack framework; host data is
    uploaded (Python integer lists become int32, as mx.array(list) does)."""
    if obj is None or isinstance(obj, DeviceArray):
        return obj
    if isinstance(obj, np.ndarray):
        return DeviceArray.from_numpy(obj)
    if hasattr(obj, "__dlpack_device__"):
        return obj
    arr = np.asarray(obj)
    if arr.dtype == np.int64:
        arr = arr.astype(np.int32)
    elif arr.dtype == np.float64:
        arr = arr.astype(np.float32)
    return DeviceArray.from_numpy(arr)


def _out_like_query(query, device_hint: int | None = None) -> DeviceArray:
    shape, _, dt, _, dev = describe(query)
    return DeviceArray.empty(shape, dt, device=dev)


def paged_attention_v1(
    query,
    key_cache,
    value_cache,
    block_tables,
    context_lens,
    num_kv_heads: int,
    scale: float,
    block_size: int,
    max_seq_len: int,
    alibi_slopes=None,
    *,
    out=None,
    stream=None,
):
    """Single-pass paged attention decode (sglang_mlx/metal_kernels.py:20-61).

    Args:
        query: [num_seqs, num_heads, head_size]
        key_cache: [num_blocks, num_kv_heads, head_size/x, block_size, x]
        value_cache: [num_blocks, num_kv_heads, head_size, block_size]
        block_tables: [num_seqs, max_num_blocks_per_seq] int32/uint32
        context_lens: [num_seqs] int32/uint32
        num_kv_heads, scale, block_size, max_seq_len: as in the reference
        alibi_slopes: optional [num_heads] float32
        out: optional preallocated output (extension); `stream`: CUDA stream (extension)

    Returns:
        [num_seqs, num_heads, head_size] in the query dtype.
    """
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    if out is None:
        out = _out_like_query(query)
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (query, "query"), (key_cache, "key_cache"),
                                           (value_cache, "value_cache"), (block_tables, "block_tables"),
                                           (context_lens, "context_lens"), (alibi_slopes, "alibi_slopes"))]
    rc = _L.kvc_paged_attention_v1(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                   int(num_kv_heads), float(scale), int(block_size), int(max_seq_len),
                                   ptrs[6][0], _stream(stream))
    _lib.check(rc)
    return out


def splitk_workspace(num_seqs: int, num_heads: int, head_size: int, max_seq_len: int,
                     partition_size: int = DEFAULT_PARTITION_SIZE, device: int | None = None):
    """(exp_sums, max_logits, tmp_out) buffers for paged_attention_v2."""
    parts = max(1, -(-int(max_seq_len) // int(partition_size)))
    es = DeviceArray.empty((num_seqs, num_heads, parts), dtypes.float32, device)
    ml = DeviceArray.empty((num_seqs, num_heads, parts), dtypes.float32, device)
    to = DeviceArray.empty((num_seqs, num_heads, parts, head_size), dtypes.float32, device)
    return es, ml, to


def paged_attention_v2(
    query,
    key_cache,
    value_cache,
    block_tables,
    context_lens,
    num_kv_heads: int,
    scale: float,
    block_size: int,
    max_seq_len: int,
    alibi_slopes=None,
    *,
    partition_size: int = DEFAULT_PARTITION_SIZE,
    workspace=None,
    out=None,
    stream=None,
    plan=None,
):
    """Split-K decode: partitions of `partition_size` tokens, each producing
    (max, sum, unnormalised output) partials, merged by a log-sum-exp reduce.
    Same arguments and result as paged_attention_v1.

    plan: a DecodePlan of make_decode_plan (same lengths, num_kv_heads,
    max_seq_len and partition_size): the partitions then run longest first and
    the last partition of a sequence merges its partials (no reduce kernel)."""
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    shape, _, _, _, dev = describe(query)
    if plan is not None and int(plan.partition_size) != int(partition_size):
        raise ValueError(f"the plan was made for partition_size {plan.partition_size}, not {partition_size}")
    if out is None:
        out = _out_like_query(query)
    if workspace is None:
        workspace = splitk_workspace(shape[0], shape[1], shape[2], max_seq_len, partition_size, dev)
    es, ml, to = workspace
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (es, "exp_sums"), (ml, "max_logits"), (to, "tmp_out"),
                                           (query, "query"), (key_cache, "key_cache"), (value_cache, "value_cache"),
                                           (block_tables, "block_tables"), (context_lens, "context_lens"),
                                           (alibi_slopes, "alibi_slopes"))]
    if plan is not None:
        pl = as_dltensor(plan.array, "plan")
        rc = _L.kvc_paged_attention_planned(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                            ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                            int(block_size), int(max_seq_len), ptrs[9][0], int(partition_size),
                                            pl[0], _stream(stream))
    else:
        rc = _L.kvc_paged_attention_v2(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                       ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                       int(block_size), int(max_seq_len), ptrs[9][0], int(partition_size),
                                       _stream(stream))
    _lib.check(rc)
    return out


def decode_plan_size(num_seqs: int, num_kv_heads: int, max_seq_len: int, partition_size: int) -> int:
    """int32 elements of a decode plan (kvc_decode_plan_size)."""
    n = int(_L.kvc_decode_plan_size(int(num_seqs), int(num_kv_heads), int(max_seq_len), int(partition_size)))
    if n < 0:
        raise ValueError(_lib.last_error() or "no decode plan covers these arguments")
    return n


class DecodePlan:
    """The work list of a planned split-K decode (kvc_decode_plan): device
    memory written on the GPU from the context lengths, reused by every layer
    of a decode step (rewrite it with make_decode_plan(..., plan=p) when the
    lengths change)."""

    def __init__(self, num_seqs: int, num_kv_heads: int, max_seq_len: int, partition_size: int,
                 device: int | None = None):
        self.num_seqs, self.num_kv_heads = int(num_seqs), int(num_kv_heads)
        self.max_seq_len, self.partition_size = int(max_seq_len), int(partition_size)
        self.array = DeviceArray.empty((decode_plan_size(num_seqs, num_kv_heads, max_seq_len, partition_size),),
                                       dtypes.int32, device)


def make_decode_plan(context_lens, num_kv_heads: int, max_seq_len: int, partition_size: int, *, plan=None,
                     stream=None) -> DecodePlan:
    """Writes (into `plan`, or a new DecodePlan) the work list of a split-K
    decode over `context_lens`: every (sequence, partition) item ordered
    longest first, and zeroed per-(sequence, KV head) arrival counters."""
    context_lens = _dev(context_lens)
    shape, _, _, _, dev = describe(context_lens)
    if plan is None:
        plan = DecodePlan(shape[0], num_kv_heads, max_seq_len, partition_size, dev)
    elif (plan.num_seqs, plan.num_kv_heads, plan.max_seq_len, plan.partition_size) != (
            int(shape[0]), int(num_kv_heads), int(max_seq_len), int(partition_size)):
        raise ValueError("plan was sized for other num_seqs / num_kv_heads / max_seq_len / partition_size")
    cl = as_dltensor(context_lens, "context_lens")
    pl = as_dltensor(plan.array, "plan")
    _lib.check(_L.kvc_decode_plan(pl[0], cl[0], int(num_kv_heads), int(max_seq_len), int(partition_size),
                                  _stream(stream)))
    return plan


def paged_attention_flash(
    query,
    key_cache,
    value_cache,
    block_tables,
    context_lens,
    num_kv_heads: int,
    scale: float,
    block_size: int,
    max_seq_len: int,
    alibi_slopes=None,
    *,
    partition_size: int | None = None,
    workspace=None,
    out=None,
    stream=None,
):
    """Decode over token-major caches: [num_blocks, block_size, kv_heads, D]
    (the reshape_and_cache_flash layout) or a token pool [slots, kv_heads, D]
    with block_size 1, whose block table rows are slot lists.  Same math and
    edge rules as paged_attention_v1.  partition_size None lets choose_decode
    pick (0 = single pass)."""
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    shape, _, _, _, dev = describe(query)
    if partition_size is None:
        # the token-major kernel keeps two CTAs per SM (16-token groups)
        partition_size = choose_decode(shape[0], num_kv_heads, max_seq_len, 16)
    if out is None:
        out = _out_like_query(query)
    ws = (None, None, None)
    if partition_size:
        ws = workspace if workspace is not None else splitk_workspace(shape[0], shape[1], shape[2], max_seq_len,
                                                                      partition_size, dev)
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (ws[0], "exp_sums"), (ws[1], "max_logits"),
                                           (ws[2], "tmp_out"), (query, "query"), (key_cache, "key_cache"),
                                           (value_cache, "value_cache"), (block_tables, "block_tables"),
                                           (context_lens, "context_lens"), (alibi_slopes, "alibi_slopes"))]
    rc = _L.kvc_paged_attention_flash(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                      ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                      int(block_size), int(max_seq_len), ptrs[9][0], int(partition_size),
                                      _stream(stream))
    _lib.check(rc)
    return out


def paged_prefill_attention(
    query,
    key_cache,
    value_cache,
    block_tables,
    qo_indptr,
    kv_lens,
    num_kv_heads: int,
    scale: float,
    block_size: int,
    *,
    max_q_len: int | None = None,
    window_size: int | None = None,
    out=None,
    stream=None,
):
    """Prefill / extend attention over a paged or token-major cache.

    query [num_tokens, num_heads, D] holds the new tokens of every sequence,
    sequence b's at rows qo_indptr[b] .. qo_indptr[b+1]-1; their K/V are already
    in the cache, whose sequence b holds kv_lens[b] tokens (prefix + new).  New
    token t of sequence b attends to cache tokens [0, prefix + t] — the
    offset-causal mask of mlx-lm's create_attention_mask that
    PooledKVCache.make_mask returns (memory_pool.py:240-270) — or, with a
    window w, to (prefix + t - w, prefix + t].  Caches: the paged layout of
    paged_attention_v1, the flash layout [nb, bs, H, D] or a token pool
    [slots, H, D] (block_size 1, block_tables rows are slot lists).
    max_q_len None: read from a host qo_indptr, else num_tokens (an upper
    bound; extra row tiles exit at once)."""
    if max_q_len is None:
        if isinstance(qo_indptr, (np.ndarray, list, tuple)):
            ind = np.asarray(qo_indptr, dtype=np.int64)
            max_q_len = int(np.max(np.diff(ind))) if ind.size > 1 else 0
        else:
            max_q_len = describe(query)[0][0]
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, qo_indptr, kv_lens = _dev(block_tables), _dev(qo_indptr), _dev(kv_lens)
    if out is None:
        out = _out_like_query(query)
    ptrs = [as_dltensor(a, n)[0] for a, n in ((out, "out"), (query, "query"), (key_cache, "key_cache"),
                                              (value_cache, "value_cache"), (block_tables, "block_tables"),
                                              (qo_indptr, "qo_indptr"), (kv_lens, "kv_lens"))]
    rc = _L.kvc_paged_prefill(*ptrs, int(num_kv_heads), float(scale), int(block_size), int(max(0, max_q_len)),
                              int(window_size or 0), _stream(stream))
    _lib.check(rc)
    return out


def cascade_partitions(num_seqs: int, num_heads: int, num_kv_heads: int, max_seq_len: int, shared_prefix_len: int,
                       block_size: int = 16, sm_count: int = 148) -> tuple[int, int]:
    """(prefix_partition_size, partition_size) for paged_attention_cascade.

    Prefix chunks are sized so that (64-row tiles of the B*G query rows) x
    (chunks) x (kv heads) is at most two per SM: one wave of the mma.sync
    prefix kernel, and at most one 128-row work item per SM for the tcgen05
    prefix kernel, which leaves the tail partitions room to run beside it.
    The tokens after the prefix form one partition when there are at most
    1024 of them, else 1024-token partitions."""
    unit = 32 * block_size // math.gcd(32, block_size)
    tiles = -(-num_seqs * (num_heads // num_kv_heads) // 64)
    chunks = max(1, 2 * sm_count // max(1, tiles * num_kv_heads))
    pp = -(-shared_prefix_len // chunks)
    pp = max(unit, -(-pp // unit) * unit)
    tail = max(0, max_seq_len - shared_prefix_len)
    pt = 1024 if tail > 1024 else max(unit, -(-tail // unit) * unit)
    return pp, pt


def cascade_workspace(num_seqs: int, num_heads: int, head_size: int, max_seq_len: int, shared_prefix_len: int,
                      prefix_partition_size: int, partition_size: int, device: int | None = None):
    """(exp_sums, max_logits, tmp_out) for paged_attention_cascade."""
    parts = -(-shared_prefix_len // prefix_partition_size)
    if max_seq_len > shared_prefix_len:
        parts += -(-(max_seq_len - shared_prefix_len) // partition_size)
    es = DeviceArray.empty((num_seqs, num_heads, parts), dtypes.float32, device)
    ml = DeviceArray.empty((num_seqs, num_heads, parts), dtypes.float32, device)
    to = DeviceArray.empty((num_seqs, num_heads, parts, head_size), dtypes.float32, device)
    return es, ml, to


def paged_attention_cascade(
    query,
    key_cache,
    value_cache,
    block_tables,
    context_lens,
    num_kv_heads: int,
    scale: float,
    block_size: int,
    max_seq_len: int,
    shared_prefix_len: int,
    *,
    prefix_partition_size: int | None = None,
    partition_size: int | None = None,
    workspace=None,
    out=None,
    stream=None,
):
    """Decode of a batch whose block tables all start with the same
    shared_prefix_len tokens (a radix-cache hit shared by every sequence): the
    prefix is attended once per KV head for all sequences together, the rest
    per sequence, merged by log-sum-exp.  Same arguments and result as
    paged_attention_v1 (no ALiBi), plus the prefix length."""
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens = _dev(block_tables), _dev(context_lens)
    shape, _, _, _, dev = describe(query)
    pp, pt = cascade_partitions(shape[0], shape[1], num_kv_heads, max_seq_len, shared_prefix_len, block_size)
    pp = prefix_partition_size or pp
    pt = partition_size or pt
    if out is None:
        out = _out_like_query(query)
    if workspace is None:
        workspace = cascade_workspace(shape[0], shape[1], shape[2], max_seq_len, shared_prefix_len, pp, pt, dev)
    es, ml, to = workspace
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (es, "exp_sums"), (ml, "max_logits"), (to, "tmp_out"),
                                           (query, "query"), (key_cache, "key_cache"), (value_cache, "value_cache"),
                                           (block_tables, "block_tables"), (context_lens, "context_lens"))]
    rc = _L.kvc_paged_attention_cascade(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                        ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                        int(block_size), int(max_seq_len), None, int(shared_prefix_len), int(pp),
                                        int(pt), _stream(stream))
    _lib.check(rc)
    return out


def choose_decode(num_seqs: int, num_kv_heads: int, max_seq_len: int, block_size: int = 16,
                  sm_count: int = 148) -> int:
    """0 for the single-pass decode, else the split-K partition size to use.

    The single-pass grid has one CTA per (sequence, kv head); the tensor-core
    kernel keeps two or three CTAs per SM, and with variable lengths it wants
    about four waves to hide the tail.  Below that, sequences are split into
    partitions.  Counting half of max_seq_len as the typical length: 2048-token
    partitions when they still give four waves, else 1024 when that gives one
    wave, else 512.  (Measured on 1/2/4/8-way head-sharded Llama-3-8B decode:
    short partitions lose more to per-CTA pipeline ramp than they gain in
    balance.)  Batches allowed to hold sequences of 8192+ tokens are split
    too: one such sequence alone in the last wave would set the launch time
    (lognormal continuous batch: 63% single pass, 91% split)."""
    slots = sm_count * (3 if block_size >= 32 else 2)
    items = num_seqs * num_kv_heads
    if max_seq_len <= 512 or (items >= 4 * slots and max_seq_len < 8192):
        return 0

    def ctas(p):
        return items * max(1, -(-max_seq_len // p)) / 2

    if ctas(2048) >= 4 * slots:
        return 2048
    if ctas(1024) >= slots:
        return 1024
    return 512


def choose_planned_partition(num_seqs: int, num_kv_heads: int, max_seq_len: int, block_size: int = 16,
                             context_lens=None, sm_count: int = 148, head_size: int = 128) -> int:
    """Partition size for the planned split-K decode (make_decode_plan).

    The plan hands out its items longest first, so the launch ends on short
    ones; what remains is to have enough items to fill the resident CTA slots
    (two per SM, three for 32-token blocks) with some to spare, without cutting
    sequences finer than that needs (each partition pays a CTA's start-up and
    its partials).  The rule: the largest of 4096, 2048, 1024, 512 tokens whose
    item count reaches 1.25 slots.  Measured on B200 (config 2 shares, 256
    sequences of U[512, 4096] tokens): 1 KV head 2048 (0.71 of HBM against 0.62
    for 1024 and 0.59 for the unplanned split-K), 2 KV heads 2048, 4 and 8 KV
    heads 4096 (0.94 / 0.985 against 0.86 / 0.92 unplanned).  `context_lens`
    (host values) gives the exact item counts; without them each sequence is
    taken as half of max_seq_len long.

    With at most two (sequence, KV head) pairs per SM (one rank's share of a
    head-sharded batch) and sequences of at most 4096 tokens (plus two blocks),
    head size 128 and blocks of up to 16 tokens, every sequence is one 4096-token
    partition: the library then runs the decode on 10-warp CTAs, one per SM
    (1 KV head of config 2: 0.77 of HBM against 0.71 with 2048-token
    partitions on 4-warp CTAs)."""
    if (head_size == 128 and block_size <= 16 and max_seq_len <= 4096 + 2 * block_size
            and int(num_seqs) * int(num_kv_heads) <= 2 * sm_count):
        return 4096
    slots = sm_count * (3 if block_size >= 32 else 2)
    if context_lens is not None:
        lens = np.asarray(context_lens, dtype=np.int64)
        lens = lens[(lens > 0) & (lens <= max_seq_len)]
    else:
        lens = np.full(int(num_seqs), max(1, int(max_seq_len) // 2), np.int64)
    unit = 32 * block_size // math.gcd(32, block_size)
    for P in (4096, 2048, 1024, 512):
        P = max(unit, P // unit * unit)
        items = int(np.sum(-(-lens // P))) * int(num_kv_heads)
        if items >= 1.25 * slots:
            return P
    return max(unit, 512 // unit * unit)


def use_split_k(num_seqs: int, num_kv_heads: int, max_seq_len: int, sm_count: int = 148,
                block_size: int = 16) -> bool:
    """True when choose_decode picks the split-K form."""
    return choose_decode(num_seqs, num_kv_heads, max_seq_len, block_size, sm_count) > 0


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads: int, scale: float,
                    block_size: int, max_seq_len: int, alibi_slopes=None, *, stream=None, out=None,
                    workspace=None, plan=None):
    """The planned split-K decode (make_decode_plan + paged_attention_v2 with
    the plan), its partition size from choose_planned_partition.  Pass a plan
    made once per decode step (every layer has the same lengths) to skip the
    plan kernel here; its partition size is then used."""
    shape, _, _, _, dev = describe(_dev(query))
    host_lens = context_lens if isinstance(context_lens, (np.ndarray, list, tuple)) else None
    if plan is None:
        psize = choose_planned_partition(shape[0], num_kv_heads, max_seq_len, block_size, host_lens,
                                         head_size=shape[2])
        context_lens = _dev(context_lens)
        plan = make_decode_plan(context_lens, num_kv_heads, max_seq_len, psize, stream=stream)
    return paged_attention_v2(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, partition_size=plan.partition_size,
                              workspace=workspace, stream=stream, out=out, plan=plan)


def paged_attention_append(query, key, value, key_cache, value_cache, slot_mapping, block_tables, context_lens,
                           num_kv_heads: int, scale: float, block_size: int, max_seq_len: int, alibi_slopes=None, *,
                           stream=None, out=None, workspace=None, plan=None):
    """A decode step's append and planned decode in one launch: the same cache
    and output as reshape_and_cache(key, value, key_cache, value_cache,
    slot_mapping) followed by paged_attention(...), for one new token per
    sequence (key/value [num_seqs, num_kv_heads, head_size] of the cache's
    dtype) whose slot slot_mapping[b] is the last position (context_lens[b] -
    1) of sequence b.  The CTA that holds each sequence's last token writes it,
    so the decode does not wait for a separate append launch.  Paged
    float16/bfloat16 caches on the tensor-core decode only (NotImplementedError
    otherwise).  Pass a plan made once per step to skip the plan kernel here."""
    query, key, value = _dev(query), _dev(key), _dev(value)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    slot_mapping = _dev(slot_mapping)
    shape, _, _, _, dev = describe(query)
    if plan is None:
        psize = choose_planned_partition(shape[0], num_kv_heads, max_seq_len, block_size, head_size=shape[2])
        plan = make_decode_plan(context_lens, num_kv_heads, max_seq_len, psize, stream=stream)
    psize = int(plan.partition_size)
    if out is None:
        out = _out_like_query(query)
    if workspace is None:
        workspace = splitk_workspace(shape[0], shape[1], shape[2], max_seq_len, psize, dev)
    es, ml, to = workspace
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (es, "exp_sums"), (ml, "max_logits"), (to, "tmp_out"),
                                           (query, "query"), (key, "key"), (value, "value"),
                                           (key_cache, "key_cache"), (value_cache, "value_cache"),
                                           (slot_mapping, "slot_mapping"), (block_tables, "block_tables"),
                                           (context_lens, "context_lens"), (alibi_slopes, "alibi_slopes"))]
    pl = as_dltensor(plan.array, "plan")
    _lib.check(_L.kvc_paged_attention_planned_append(
        ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0], ptrs[6][0], ptrs[7][0], ptrs[8][0],
        ptrs[9][0], ptrs[10][0], ptrs[11][0], int(num_kv_heads), float(scale), int(block_size), int(max_seq_len),
        ptrs[12][0], psize, pl[0], _stream(stream)))
    return out


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, *, stream=None):
    """Scatter-write new KV tokens into the paged cache (metal_kernels.py:64-74).

    The caches are updated in place and returned, as the reference's outputs
    alias its inputs (mlx_cache.cpp:65-66).
    """
    key, value, slot_mapping = _dev(key), _dev(value), _dev(slot_mapping)
    ptrs = [as_dltensor(a, n) for a, n in ((key, "key"), (value, "value"), (key_cache, "key_cache"),
                                           (value_cache, "value_cache"), (slot_mapping, "slot_mapping"))]
    _lib.check(_L.kvc_reshape_and_cache(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], _stream(stream)))
    return [key_cache, value_cache]


def reshape_and_cache_flash(key, value, key_cache, value_cache, slot_mapping, *, stream=None):
    """Flash-layout append ([num_blocks, block_size, H, D] caches, bindings.cpp:82-95)."""
    key, value, slot_mapping = _dev(key), _dev(value), _dev(slot_mapping)
    ptrs = [as_dltensor(a, n) for a, n in ((key, "key"), (value, "value"), (key_cache, "key_cache"),
                                           (value_cache, "value_cache"), (slot_mapping, "slot_mapping"))]
    _lib.check(_L.kvc_reshape_and_cache_flash(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0],
                                              _stream(stream)))
    return [key_cache, value_cache]


def gather_kv(k_buffer, v_buffer, indices, *, k_out=None, v_out=None, stream=None):
    """out[0, h, t, :] = buffer[indices[t], h, :] for K and V (MHATokenPool.fetch)."""
    kshape, _, dt, _, dev = describe(k_buffer)
    idx = _dev(indices) if not isinstance(indices, (list, tuple)) else DeviceArray.from_numpy(
        np.asarray(indices, dtype=np.int32), device=dev)
    T = describe(idx)[0][0]
    H, D = kshape[-2], kshape[-1]
    if k_out is None:
        k_out = DeviceArray.empty((1, H, T, D), dt, device=dev)
    if v_out is None:
        v_out = DeviceArray.empty((1, H, T, D), dt, device=dev)
    ptrs = [as_dltensor(a, n) for a, n in ((k_out, "k_out"), (v_out, "v_out"), (k_buffer, "k_buffer"),
                                           (v_buffer, "v_buffer"), (idx, "indices"))]
    _lib.check(_L.kvc_gather_kv(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], _stream(stream)))
    return k_out, v_out


def _mapping(block_mapping):
    """A block mapping as an array libkvcache accepts: device arrays and
    DLPack producers pass through, anything else becomes a host int64 array."""
    if isinstance(block_mapping, DeviceArray) or hasattr(block_mapping, "__dlpack__"):
        if isinstance(block_mapping, np.ndarray):
            return np.ascontiguousarray(block_mapping)
        return block_mapping
    return np.ascontiguousarray(np.asarray(block_mapping, dtype=np.int64))


# FP8 formats.  "e4m3" / "e5m2" encode exactly as the reference's float8.metal
# code does (values past E4M3's last finite exponent go down its subnormal
# branch, a subnormal's carry into the smallest normal is dropped; +-Inf where
# that code's shift is undefined).  "e4m3-sat" / "e5m2-sat" encode with the
# behaviour that file's comment states instead: +-Inf past the largest finite
# value and the carry kept.  Decoding is the same for both.
_FP8 = {"e4m3": 0, "e5m2": 1, "e4m3-sat": 2, "e5m2-sat": 3}


def _fp8_format(name: str) -> int:
    if name not in _FP8:
        raise ValueError(f"fp8_format must be one of {sorted(_FP8)}")
    return _FP8[name]


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping, k_scale: float = 1.0,
                          v_scale: float = 1.0, fp8_format: str = "e4m3", *, stream=None):
    """reshape_and_cache into one-byte (uint8) caches: each value is stored as
    encode(x / scale) in the float8.metal code of `fp8_format`.  Caches are
    [nb, kv_heads, D/16, bs, 16] and [nb, kv_heads, D, bs]."""
    ptrs = [as_dltensor(_dev(a), n) for a, n in ((key, "key"), (value, "value"), (key_cache, "key_cache"),
                                                 (value_cache, "value_cache"), (slot_mapping, "slot_mapping"))]
    _lib.check(_L.kvc_reshape_and_cache_fp8(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0],
                                            float(k_scale), float(v_scale), _fp8_format(fp8_format), _stream(stream)))
    return [key_cache, value_cache]


def paged_attention_fp8(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads: int, scale: float,
                        block_size: int, max_seq_len: int, alibi_slopes=None, *, k_scale: float = 1.0,
                        v_scale: float = 1.0, fp8_format: str = "e4m3", partition_size: int | None = None,
                        workspace=None, out=None, stream=None, plan=None):
    """paged_attention_v1 over one-byte caches written by reshape_and_cache_fp8
    (values decode(code) * scale).  partition_size None lets choose_decode pick
    (0 = single pass); with a DecodePlan (make_decode_plan) the planned split-K
    runs with the plan's partition size."""
    if plan is not None:
        if partition_size not in (None, plan.partition_size):
            raise ValueError(f"the plan was made for partition_size {plan.partition_size}, not {partition_size}")
        partition_size = plan.partition_size
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    shape, _, _, _, dev = describe(query)
    if partition_size is None:
        partition_size = choose_decode(shape[0], num_kv_heads, max_seq_len, 16 if block_size <= 16 else 32)
    if out is None:
        out = _out_like_query(query)
    ws = (None, None, None)
    if partition_size:
        ws = workspace if workspace is not None else splitk_workspace(shape[0], shape[1], shape[2], max_seq_len,
                                                                      partition_size, dev)
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (ws[0], "exp_sums"), (ws[1], "max_logits"),
                                           (ws[2], "tmp_out"), (query, "query"), (key_cache, "key_cache"),
                                           (value_cache, "value_cache"), (block_tables, "block_tables"),
                                           (context_lens, "context_lens"), (alibi_slopes, "alibi_slopes"))]
    if plan is not None:
        pl = as_dltensor(plan.array, "plan")
        rc = _L.kvc_paged_attention_fp8_planned(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0],
                                                ptrs[5][0], ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads),
                                                float(scale), int(block_size), int(max_seq_len), ptrs[9][0],
                                                float(k_scale), float(v_scale), _fp8_format(fp8_format),
                                                int(partition_size), pl[0], _stream(stream))
    else:
        rc = _L.kvc_paged_attention_fp8(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                        ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                        int(block_size), int(max_seq_len), ptrs[9][0], float(k_scale),
                                        float(v_scale), _fp8_format(fp8_format), int(partition_size),
                                        _stream(stream))
    _lib.check(rc)
    return out


def convert_fp8(dst, src, scale: float = 1.0, fp8_format: str = "e4m3", *, stream=None):
    """convert_fp8_kernel (convert_fp8.metal:13-80): uint8 codes <-> float
    arrays of the same shape (quantise encode(x / scale), dequantise
    decode(code) * scale, rescale codes, or scale floats).  Returns dst."""
    d, dk = as_dltensor(_dev(dst), "dst")
    s, sk = as_dltensor(_dev(src), "src")
    _lib.check(_L.kvc_convert_fp8(d, s, float(scale), _fp8_format(fp8_format), _stream(stream)))
    del dk, sk
    return dst


def copy_blocks(key_caches, value_caches, block_mapping, *, stream=None):
    """Copy blocks within the cache (metal_kernels.py:77-85): for every layer and
    every pair (src, dst) of `block_mapping` ([num_pairs, 2]), block dst of the
    layer's key and value caches is overwritten with block src.  The caches are
    updated in place; returns (key_caches, value_caches) as the reference does."""
    keys, vals = [_dev(x) for x in key_caches], [_dev(x) for x in value_caches]
    kd = [as_dltensor(x, f"key_caches[{i}]") for i, x in enumerate(keys)]
    vd = [as_dltensor(x, f"value_caches[{i}]") for i, x in enumerate(vals)]
    karr = (DLTensor * max(1, len(kd)))(*[p.contents for p, _ in kd])
    varr = (DLTensor * max(1, len(vd)))(*[p.contents for p, _ in vd])
    m, mkeep = as_dltensor(_mapping(block_mapping), "block_mapping")
    _lib.check(_L.kvc_copy_blocks(ctypes.cast(karr, ctypes.c_void_p), len(kd), ctypes.cast(varr, ctypes.c_void_p),
                                  len(vd), m, _stream(stream)))
    del kd, vd, mkeep
    return keys, vals


def swap_blocks(src, dst, block_mapping, *, stream=None):
    """Blit blocks between two buffers (metal_kernels.py:88-96): block dst of
    `dst` is overwritten with block src of `src` for every pair.  Either side
    may be device memory or host memory (a HostBuffer, pinned, or a NumPy
    array); returns `dst`, updated in place."""
    def side(x):
        return x if isinstance(x, (HostBuffer, np.ndarray)) else _dev(x)

    dst = side(dst)
    s, skeep = as_dltensor(side(src), "src")
    d, dkeep = as_dltensor(dst, "dst")
    m, mkeep = as_dltensor(_mapping(block_mapping), "block_mapping")
    _lib.check(_L.kvc_swap_blocks(s, d, m, _stream(stream)))
    del skeep, dkeep, mkeep
    return dst


def get_max_shared_memory_per_block_device_attribute(device_id: int = 0) -> int:
    """bindings.cpp:125-133 / mlx_device.cpp:16-20."""
    v = ctypes.c_int64(0)
    _lib.check(_L.kvc_get_max_shared_memory_per_block_device_attribute(int(device_id), ctypes.byref(v)))
    return int(v.value)


def get_device_attribute(attribute: int, device_id: int = 0) -> int:
    """bindings.cpp:125-128; a cudaDeviceAttr value (mlx_device.cpp:12-14 throws on Metal)."""
    v = ctypes.c_int64(0)
    _lib.check(_L.kvc_get_device_attribute(int(attribute), int(device_id), ctypes.byref(v)))
    return int(v.value)


def synchronize() -> None:
    _lib.synchronize()


__all__ = [
    "paged_attention_v1",
    "paged_attention_v2",
    "paged_attention",
    "reshape_and_cache",
    "reshape_and_cache_flash",
    "gather_kv",
    "copy_blocks",
    "swap_blocks",
    "splitk_workspace",
    "use_split_k",
    "get_max_shared_memory_per_block_device_attribute",
    "get_device_attribute",
    "synchronize",
    "asarray",
]
