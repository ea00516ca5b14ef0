"""KV memory pool on B200, API-compatible with
sglang_mlx/srt/mem_cache/memory_pool.py.

- TokenPoolAllocator: the same LIFO free list (memory_pool.py:27-68); a fresh
  pool hands out slots in descending order and slot 0 is never allocated.
- MHATokenPool: per-layer K/V device buffers of shape (pool_size + 1, H, D)
  (memory_pool.py:76-108).  `store` is one libkvcache append launch that reads
  the (1, H, S, D) input through its strides (no transpose copy); `fetch` is one
  gather launch writing (1, H, T, D) (memory_pool.py:117-159).
- PooledKVCache: the per-request adapter (memory_pool.py:167-269), unchanged
  in behaviour.

Beyond the reference: the decode its pool leaves as a TODO
(memory_pool.py:110-112) — attention straight on the scattered pool slots,
with no per-layer gather.  MHATokenPool.decode runs it for a batch of slot
lists; PooledKVCache.update_and_attend is update_and_fetch followed by the
attention, for single-token decode, in two launches (append, decode).
"""

from __future__ import annotations

import ctypes

import numpy as np

from ... import _lib, dtypes
from ...device_array import DeviceArray, _stream
from ...dlpack import as_dltensor, describe, make_dltensor

_L = _lib.lib


class TokenPoolAllocator:
    """Free list of the pool's token slots, handed out last-in first-out.

    Slot 0 is the padding slot that block tables point at for unused
    positions; it is never handed out, so a fresh pool gives n, n-1, ..., 1
    for alloc(n).

    page_size > 1 (the reference's radix cache is page-size-1 only,
    radix_cache.py:11, cache_init_params.py:16) hands out whole pages: page p
    holds slots p * page_size + 1 .. (p + 1) * page_size, so a request's slots
    fill its pages in order and a decode can read them page by page
    (MHATokenPool.decode_pages) instead of slot by slot.  alloc(n) takes
    ceil(n / page_size) free pages and returns their first n slots;
    alloc_extend(last_slot, n) continues inside last_slot's page before taking
    new ones; a page returns to the free list once every slot handed out from
    it has been freed.
    """

    def __init__(self, pool_size: int, page_size: int = 1):
        if pool_size <= 0:
            raise ValueError(f"pool_size must be positive, got {pool_size}")
        if page_size <= 0 or pool_size % page_size:
            raise ValueError(f"pool_size ({pool_size}) must be a positive multiple of page_size ({page_size})")
        self._pool_size = pool_size
        self.page_size = page_size
        if page_size == 1:
            # Slots 1..pool_size are allocatable; kept as a stack (memory_pool.py:38).
            self._free_slots: list[int] = list(range(pool_size, 0, -1))
        else:
            self._num_pages = pool_size // page_size
            self._free_pages: list[int] = list(range(self._num_pages - 1, -1, -1))
            self._used = [0] * self._num_pages  # slots handed out per page

    def _page_slots(self, page: int) -> range:
        return range(page * self.page_size + 1, (page + 1) * self.page_size + 1)

    def _take_pages(self, n_pages: int) -> list[int]:
        if n_pages > len(self._free_pages):
            raise MemoryError(f"Cannot allocate {n_pages} pages: only {len(self._free_pages)} available")
        pages = self._free_pages[-n_pages:][::-1]
        del self._free_pages[-n_pages:]
        return pages

    def alloc(self, n: int) -> list[int]:
        """Pops the last *n* free slots; MemoryError if fewer are free.  With
        pages: the first n slots of ceil(n / page_size) free pages."""
        if n <= 0:
            return []
        if self.page_size == 1:
            if n > len(self._free_slots):
                raise MemoryError(f"Cannot allocate {n} slots: only {len(self._free_slots)} available")
            allocated = self._free_slots[-n:]
            del self._free_slots[-n:]
            return allocated
        pages = self._take_pages(-(-n // self.page_size))
        out = []
        for pg in pages:
            take = min(self.page_size, n - len(out))
            out.extend(self._page_slots(pg)[:take])
            self._used[pg] = take
        return out

    def alloc_extend(self, last_slot: int, n: int) -> list[int]:
        """n more slots for a request whose last slot is `last_slot`: the rest of
        its page first (pages), then new pages.  Page size 1: alloc(n)."""
        if self.page_size == 1 or n <= 0:
            return self.alloc(n)
        page = (int(last_slot) - 1) // self.page_size
        room = (page + 1) * self.page_size - int(last_slot)
        take = min(room, n)
        if take and not 0 <= page < self._num_pages:
            raise ValueError(f"slot {last_slot} is not in the pool")
        out = list(range(int(last_slot) + 1, int(last_slot) + 1 + take))
        if take:
            self._used[page] += take
        if n > take:
            out += self.alloc(n - take)
        return out

    def free(self, indices: list[int]) -> None:
        """Returns *indices* to the free list (pages: a page once all its handed-out slots are back)."""
        if self.page_size == 1:
            self._free_slots.extend(indices)
            return
        for i in indices:
            pg = (int(i) - 1) // self.page_size
            self._used[pg] -= 1
            if self._used[pg] == 0:
                self._free_pages.append(pg)

    @property
    def available_size(self) -> int:
        if self.page_size == 1:
            return len(self._free_slots)
        return len(self._free_pages) * self.page_size

    def clear(self) -> None:
        """Resets all slots to free."""
        if self.page_size == 1:
            self._free_slots = list(range(self._pool_size, 0, -1))
        else:
            self._free_pages = list(range(self._num_pages - 1, -1, -1))
            self._used = [0] * self._num_pages


def slots_to_pages(slots, page_size: int):
    """The page table of a slot list that fills pages in order (TokenPoolAllocator
    with page_size > 1), or None when the slots are not page-aligned: slot i of
    the list must be page_i * page_size + 1 + i % page_size."""
    s = np.asarray(slots, dtype=np.int64)
    if page_size <= 1 or s.size == 0:
        return None
    pos = np.arange(s.size)
    pages = (s - 1) // page_size
    if np.any((s - 1) % page_size != pos % page_size):
        return None
    head = pages[::page_size]
    if np.any(pages != np.repeat(head, page_size)[: s.size]):
        return None
    return head.astype(np.int32)


def _index_array(indices, device: int) -> DeviceArray:
    if isinstance(indices, DeviceArray):
        return indices
    if hasattr(indices, "__dlpack_device__") and not isinstance(indices, np.ndarray):
        return indices
    arr = np.asarray(indices, dtype=np.int64)
    if arr.size and (arr.min() < np.iinfo(np.int32).min or arr.max() > np.iinfo(np.int32).max):
        return DeviceArray.from_numpy(arr, device=device)
    return DeviceArray.from_numpy(arr.astype(np.int32), device=device)


class MHATokenPool:
    """The K and V device buffers of every layer, allocated once up front.

    Each layer holds one ``(pool_size + 1, n_kv_heads, head_dim)`` buffer for K
    and one for V, a token's row per slot (slot 0 stays padding).  Attention
    code sees ``(1, n_kv_heads, S, head_dim)`` arrays: store takes that shape
    and fetch returns it; the decode reads the slots in place.
    """

    def __init__(self, pool_size: int, num_layers: int, n_kv_heads: int, head_dim: int,
                 dtype=dtypes.float16, device: int | None = None, page_size: int = 1):
        if page_size <= 0 or pool_size % page_size:
            raise ValueError(f"pool_size ({pool_size}) must be a positive multiple of page_size ({page_size})")
        self.pool_size = pool_size
        self.page_size = page_size
        self.num_layers = num_layers
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.dtype = dtypes.canonical(dtype)
        self.device = _lib.current_device() if device is None else int(device)
        shape = (pool_size + 1, n_kv_heads, head_dim)  # +1 for slot 0 padding
        self.k_buffer: list[DeviceArray] = [DeviceArray.zeros(shape, self.dtype, self.device)
                                            for _ in range(num_layers)]
        self.v_buffer: list[DeviceArray] = [DeviceArray.zeros(shape, self.dtype, self.device)
                                            for _ in range(num_layers)]

    def store(self, layer_idx: int, indices, keys, values, *, stream=None) -> None:
        """Writes KV data into the pool at the given slot indices.

        Args:
            layer_idx: Which transformer layer.
            indices: Pool slot indices, length S (list, NumPy or device array).
            keys: ``(1, n_kv_heads, S, head_dim)``; values: same shape.
        """
        kshape, kstr, kdt, _, kdev = describe(keys)
        vshape, vstr, vdt, _, _ = describe(values)
        if len(kshape) != 4 or kshape[0] != 1 or tuple(vshape) != tuple(kshape):
            raise ValueError("keys and values must have shape (1, n_kv_heads, S, head_dim)")
        S = kshape[2]
        if S == 0:
            return
        idx = _index_array(indices, kdev)
        if describe(idx)[0][0] != S:
            raise ValueError(f"store: {describe(idx)[0][0]} indices for {S} tokens")
        kptr, kkeep = as_dltensor(keys, "keys")
        vptr, vkeep = as_dltensor(values, "values")
        # (1, H, S, D) read as (S, H, D) through strides: the transpose of
        # memory_pool.py:131-133 without a copy.
        kt, kk = make_dltensor(kptr.contents.data + kptr.contents.byte_offset, (S, kshape[1], kshape[3]),
                               (kstr[2], kstr[1], kstr[3]), kdt, kptr.contents.device.device_id)
        vt, vk = make_dltensor(vptr.contents.data + vptr.contents.byte_offset, (S, vshape[1], vshape[3]),
                               (vstr[2], vstr[1], vstr[3]), vdt, vptr.contents.device.device_id)
        ip, ikeep = as_dltensor(idx, "indices")
        kb = self.k_buffer[layer_idx]._dltensor()
        vb = self.v_buffer[layer_idx]._dltensor()
        _lib.check(_L.kvc_reshape_and_cache_flash(ctypes.pointer(kt), ctypes.pointer(vt), ctypes.pointer(kb),
                                                  ctypes.pointer(vb), ip, _stream(stream)))
        del kkeep, vkeep, kk, vk, ikeep

    def fetch(self, layer_idx: int, indices, *, stream=None, k_out=None, v_out=None):
        """Gathers KV data from the pool in ``(1, n_kv_heads, T, head_dim)`` format."""
        idx = _index_array(indices, self.device)
        T = describe(idx)[0][0]
        shape = (1, self.n_kv_heads, T, self.head_dim)
        if k_out is None:
            k_out = DeviceArray.empty(shape, self.dtype, self.device)
        if v_out is None:
            v_out = DeviceArray.empty(shape, self.dtype, self.device)
        if T == 0:
            return k_out, v_out
        ptrs = [as_dltensor(a, n) for a, n in ((k_out, "k_out"), (v_out, "v_out"), (self.k_buffer[layer_idx], "k"),
                                               (self.v_buffer[layer_idx], "v"), (idx, "indices"))]
        _lib.check(_L.kvc_gather_kv(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], _stream(stream)))
        return k_out, v_out

    def decode(self, layer_idx: int, queries, slot_tables, context_lens, scale: float | None = None, *,
               max_seq_len: int | None = None, alibi_slopes=None, partition_size: int | None = None,
               out=None, stream=None):
        """Single-token attention of a batch straight on the pool's slots.

        Args:
            queries: ``(B, n_heads, head_dim)``, n_heads a multiple of n_kv_heads.
            slot_tables: ``(B, max_len)`` int32 slot lists (sequence b attends
                to slots ``slot_tables[b, :context_lens[b]]``, in order).
            context_lens: ``(B,)`` int32.
            scale: softmax scale, default ``head_dim ** -0.5``.
        Returns ``(B, n_heads, head_dim)`` in the pool dtype.
        """
        from ... import metal_kernels as mk

        tshape = describe(slot_tables)[0] if not isinstance(slot_tables, (list, np.ndarray)) \
            else np.asarray(slot_tables).shape
        if max_seq_len is None:
            max_seq_len = max(1, int(tshape[1]))
        if scale is None:
            scale = self.head_dim ** -0.5
        return mk.paged_attention_flash(queries, self.k_buffer[layer_idx], self.v_buffer[layer_idx], slot_tables,
                                        context_lens, self.n_kv_heads, scale, 1, max_seq_len, alibi_slopes,
                                        partition_size=partition_size, out=out, stream=stream)


    def page_view(self, layer_idx: int):
        """K and V of `layer_idx` as [pool_size / page_size, page_size, n_kv_heads,
        head_dim] pages (the reshape_and_cache_flash layout), page p being slots
        p * page_size + 1 .. (p + 1) * page_size: a view from slot 1, no copy."""
        ps = self.page_size
        if ps <= 1:
            raise ValueError("page_view needs a pool made with page_size > 1")
        shape = (self.pool_size // ps, ps, self.n_kv_heads, self.head_dim)
        return (self.k_buffer[layer_idx][1:].reshape(*shape), self.v_buffer[layer_idx][1:].reshape(*shape))

    def decode_pages(self, layer_idx: int, queries, page_tables, context_lens, scale: float | None = None, *,
                     max_seq_len: int | None = None, alibi_slopes=None, partition_size: int | None = None,
                     out=None, stream=None):
        """decode() over page tables: sequence b's token t is slot
        page_tables[b, t // page_size] * page_size + 1 + t % page_size (slots from
        TokenPoolAllocator(page_size=...)).  Pages of 16k tokens are read with
        one tensor copy per 16 tokens and head."""
        from ... import metal_kernels as mk

        ps = self.page_size
        tshape = describe(page_tables)[0] if not isinstance(page_tables, (list, np.ndarray)) \
            else np.asarray(page_tables).shape
        if max_seq_len is None:
            max_seq_len = max(1, int(tshape[1]) * ps)
        if scale is None:
            scale = self.head_dim ** -0.5
        kv, vv = self.page_view(layer_idx)
        return mk.paged_attention_flash(queries, kv, vv, page_tables, context_lens, self.n_kv_heads, scale, ps,
                                        max_seq_len, alibi_slopes, partition_size=partition_size, out=out,
                                        stream=stream)


class PooledKVCache:
    """Adapter that makes the shared KV pool look like a per-request KV cache.

    Models call ``cache.update_and_fetch(keys, values)`` in each attention
    layer: the new tokens are stored into the pool and all (prefix + new)
    tokens are gathered back contiguously.
    """

    def __init__(self, pool: MHATokenPool, layer_idx: int):
        self._pool = pool
        self._layer_idx = layer_idx
        self._prefix_indices: list[int] = []
        self._new_indices: list[int] = []
        self._store_offset: int = 0

    def set_indices(self, prefix_indices: list[int], new_indices: list[int]) -> None:
        """Configures this layer's slots before a forward pass (memory_pool.py:186-195)."""
        self._prefix_indices = list(prefix_indices)
        self._new_indices = list(new_indices)
        self._store_offset = 0

    @property
    def offset(self) -> int:
        """RoPE position offset of the new tokens (memory_pool.py:197-204)."""
        return len(self._prefix_indices)

    def _all_indices(self) -> list[int]:
        return self._prefix_indices + self._new_indices[: self._store_offset]

    def _store_new(self, keys, values, stream=None) -> None:
        n_new = describe(keys)[0][2]
        store_indices = self._new_indices[self._store_offset: self._store_offset + n_new]
        self._store_offset += n_new
        self._pool.store(self._layer_idx, store_indices, keys, values, stream=stream)

    def update_and_fetch(self, keys, values):
        """Stores new KV and gathers all (prefix + new) KV (memory_pool.py:206-234)."""
        self._store_new(keys, values)
        return self._pool.fetch(self._layer_idx, self._all_indices())

    def update_and_attend(self, queries, keys, values, scale: float | None = None, *, window_size: int | None = None,
                          stream=None):
        """Stores the new tokens' KV and attends over prefix + new slots on the
        pool itself, without the gather of update_and_fetch: the result mlx SDPA
        gives on update_and_fetch's K/V under make_mask's mask
        (memory_pool.py:205-270).  One new token runs the decode kernel; more
        (prefill / extend) or a sliding window run the prefill kernel, where new
        token t sees slots [0, offset + t] (the last `window_size` of them).

        Args:
            queries: ``(1, n_heads, N, head_dim)``; keys, values:
                ``(1, n_kv_heads, N, head_dim)`` (mlx-lm format).
        Returns ``(1, n_heads, N, head_dim)``.
        """
        qshape, qstr, qdt, _, qdev = describe(queries)
        kshape = describe(keys)[0]
        if len(qshape) != 4 or qshape[0] != 1 or len(kshape) != 4 or kshape[2] != qshape[2]:
            raise ValueError("update_and_attend takes queries (1, H, N, D) and keys/values (1, H_kv, N, D) "
                             "with the same N")
        N = qshape[2]
        self._store_new(keys, values, stream=stream)
        slots = np.asarray(self._all_indices(), dtype=np.int32)[None, :]
        T = slots.shape[1]
        qptr, qkeep = as_dltensor(queries, "queries")
        # the queries as [N, H, D] rows (a strided view, no copy)
        qt, qk = make_dltensor(qptr.contents.data + qptr.contents.byte_offset, (N, qshape[1], qshape[3]),
                               (qstr[2], qstr[1], qstr[3]), qdt, qptr.contents.device.device_id)
        out = DeviceArray.empty((N, qshape[1], qshape[3]), qdt, qdev)
        lens = DeviceArray.from_numpy(np.array([T], dtype=np.int32), device=qdev)
        tables = DeviceArray.from_numpy(slots, device=qdev)
        if scale is None:
            scale = self._pool.head_dim ** -0.5
        from ... import metal_kernels as mk

        kbuf, vbuf = self._pool.k_buffer[self._layer_idx], self._pool.v_buffer[self._layer_idx]
        if N == 1 and not window_size:
            # slots that fill whole pages in order (a page-granular allocator) are read page by page
            ps = getattr(self._pool, "page_size", 1)
            pages = slots_to_pages(slots[0], ps)
            bs, msl = 1, T
            if pages is not None:
                kbuf, vbuf = self._pool.page_view(self._layer_idx)
                tables = DeviceArray.from_numpy(pages[None, :], device=qdev)
                bs, msl = ps, len(pages) * ps
            ws = (None, None, None)
            psize = mk.choose_decode(1, self._pool.n_kv_heads, msl, 16)
            if psize:
                psize = -(-psize // bs) * bs
                ws = mk.splitk_workspace(1, qshape[1], qshape[3], msl, psize, qdev)
            ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (ws[0], "exp_sums"), (ws[1], "max_logits"),
                                                   (ws[2], "tmp_out"), (kbuf, "k"), (vbuf, "v"), (tables, "tables"),
                                                   (lens, "lens"))]
            _lib.check(_L.kvc_paged_attention_flash(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0],
                                                    ctypes.pointer(qt), ptrs[4][0], ptrs[5][0], ptrs[6][0],
                                                    ptrs[7][0], self._pool.n_kv_heads, float(scale), bs, msl, None,
                                                    int(psize), _stream(stream)))
        else:
            indptr = DeviceArray.from_numpy(np.array([0, N], dtype=np.int32), device=qdev)
            ptrs = [as_dltensor(a, n) for a, n in ((out, "out"), (kbuf, "k"), (vbuf, "v"), (tables, "tables"),
                                                   (indptr, "qo_indptr"), (lens, "kv_lens"))]
            _lib.check(_L.kvc_paged_prefill(ptrs[0][0], ctypes.pointer(qt), ptrs[1][0], ptrs[2][0], ptrs[3][0],
                                            ptrs[4][0], ptrs[5][0], self._pool.n_kv_heads, float(scale), 1, N,
                                            int(window_size or 0), _stream(stream)))
        del qkeep, qk, ptrs
        # (N, H, D) -> a (1, H, N, D) view
        return out.transpose(1, 0, 2).expand_dims(0)

    @property
    def state(self):
        """Current cached KV, or (None, None) when empty (memory_pool.py:236-242)."""
        all_indices = self._all_indices()
        if not all_indices:
            return None, None
        return self._pool.fetch(self._layer_idx, all_indices)

    def make_mask(self, N: int, return_array: bool = False, window_size: int | None = None):
        """Attention mask of the mlx-lm convention the reference delegates to
        (memory_pool.py:244-269; behaviour pinned by test_memory_pool.py:253-330):
        None for single-token decode, "causal" for plain prefill, else a boolean
        (N, offset + N) array."""
        if N == 1:
            return None
        if not return_array and window_size is None:
            return "causal"
        offset = self.offset
        rows = np.arange(offset, offset + N)[:, None]
        cols = np.arange(offset + N)[None, :]
        mask = cols <= rows
        if window_size is not None:
            mask &= cols > rows - window_size
        return mask
