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
):
    """Split-K decode: partitions of `partition_size` tokens, each producing
    (max, sum, unnormalised output) partials, merged by a log-sum-exp reduce.
    Same arguments and result as paged_attention_v1."""
    query, key_cache, value_cache = _dev(query), _dev(key_cache), _dev(value_cache)
    block_tables, context_lens, alibi_slopes = _dev(block_tables), _dev(context_lens), _dev(alibi_slopes)
    shape, _, _, _, dev = describe(query)
    if out is None:
        out = _out_like_query(query)
    if workspace is None:
        workspace = splitk_workspace(shape[0], shape[1], shape[2], max_seq_len, partition_size, dev)
    es, ml, to = workspace
    ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (es, "exp_sums"), (ml, "max_logits"), (to, "tmp_out"),
                                           (query, "query"), (key_cache, "key_cache"), (value_cache, "value_cache"),
                                           (block_tables, "block_tables"), (context_lens, "context_lens"),
                                           (alibi_slopes, "alibi_slopes"))]
    rc = _L.kvc_paged_attention_v2(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0],
                                   ptrs[6][0], ptrs[7][0], ptrs[8][0], int(num_kv_heads), float(scale),
                                   int(block_size), int(max_seq_len), ptrs[9][0], int(partition_size),
                                   _stream(stream))
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


def use_split_k(num_seqs: int, num_kv_heads: int, max_seq_len: int, sm_count: int = 148,
                block_size: int = 16) -> bool:
    """True when choose_decode picks the split-K form."""
    return choose_decode(num_seqs, num_kv_heads, max_seq_len, block_size, sm_count) > 0


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads: int, scale: float,
                    block_size: int, max_seq_len: int, alibi_slopes=None, *, stream=None, out=None,
                    workspace=None):
    """Single-pass or split-K decode, whichever choose_decode picks for the shape."""
    shape, _, _, _, _ = describe(_dev(query))
    psize = choose_decode(shape[0], num_kv_heads, max_seq_len, block_size)
    if psize:
        return paged_attention_v2(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                                  block_size, max_seq_len, alibi_slopes, partition_size=psize, workspace=workspace,
                                  stream=stream, out=out)
    return paged_attention_v1(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                              block_size, max_seq_len, alibi_slopes, stream=stream, out=out)


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
