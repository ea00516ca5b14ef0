"""KV pool: allocator (CPU), MHATokenPool / PooledKVCache on the device (GPU).

Mirrors the reference's tests/test_memory_pool.py (allocator, store/fetch
round trips, cache adapter) and pins store/fetch against the reference pool
run by tests/golden/make_golden.py."""

import numpy as np
import pytest

from sglang_mlx_b200.srt.mem_cache.memory_pool import MHATokenPool, PooledKVCache, TokenPoolAllocator


# ---- TokenPoolAllocator (test_memory_pool.py:17-79) ------------------------------

class TestTokenPoolAllocator:
    def test_basic_alloc_free(self):
        alloc = TokenPoolAllocator(pool_size=10)
        assert alloc.available_size == 10
        slots = alloc.alloc(3)
        assert len(slots) == 3 and alloc.available_size == 7
        alloc.free(slots)
        assert alloc.available_size == 10

    def test_slot_zero_reserved(self):
        alloc = TokenPoolAllocator(pool_size=100)
        all_slots = alloc.alloc(100)
        assert 0 not in all_slots and all(s >= 1 for s in all_slots)

    def test_alloc_zero_returns_empty(self):
        alloc = TokenPoolAllocator(pool_size=5)
        assert alloc.alloc(0) == [] and alloc.available_size == 5

    def test_alloc_overflow_raises(self):
        with pytest.raises(MemoryError, match="Cannot allocate"):
            TokenPoolAllocator(pool_size=5).alloc(6)

    def test_alloc_exact_capacity(self):
        alloc = TokenPoolAllocator(pool_size=5)
        assert len(alloc.alloc(5)) == 5 and alloc.available_size == 0

    def test_free_then_realloc(self):
        alloc = TokenPoolAllocator(pool_size=5)
        alloc.free(alloc.alloc(3))
        assert len(alloc.alloc(5)) == 5

    def test_clear_resets(self):
        alloc = TokenPoolAllocator(pool_size=10)
        alloc.alloc(10)
        alloc.clear()
        assert alloc.available_size == 10

    def test_invalid_pool_size(self):
        for n in (0, -1):
            with pytest.raises(ValueError):
                TokenPoolAllocator(pool_size=n)

    def test_no_duplicate_slots(self):
        alloc = TokenPoolAllocator(pool_size=50)
        s = alloc.alloc(20) + alloc.alloc(20)
        assert len(set(s)) == len(s)

    def test_order_matches_reference(self, golden):
        """Exact LIFO order of the reference allocator (descending on a fresh pool)."""
        alloc = TokenPoolAllocator(pool_size=40)
        a1 = alloc.alloc(5)
        a2 = alloc.alloc(7)
        alloc.free(a1[1:3])
        a3 = alloc.alloc(4)
        np.testing.assert_array_equal(np.array(a1 + [-1] + a2 + [-1] + a3), golden["pool/alloc_seq"])
        assert alloc.available_size == int(golden["pool/available"])


# ---- make_mask (test_memory_pool.py:253-330) --------------------------------------

class _NoPool:
    pass


class TestMask:
    def cache(self, prefix, new):
        c = PooledKVCache(_NoPool(), 0)
        c.set_indices(prefix_indices=prefix, new_indices=new)
        return c

    def test_decode_returns_none(self):
        assert self.cache([1, 2, 3], [4]).make_mask(N=1) is None
        assert self.cache([1, 2, 3, 4, 5], [6]).make_mask(N=1, return_array=True) is None

    def test_prefill_causal(self):
        assert self.cache([], [1, 2, 3, 4]).make_mask(N=4) == "causal"
        assert self.cache([1, 2, 3], [4, 5]).make_mask(N=2) == "causal"

    def test_window(self):
        m = self.cache([], [1, 2, 3]).make_mask(N=3, window_size=2)
        assert m.shape == (3, 3) and not m[2, 0] and m[2, 1] and m[2, 2]

    def test_return_array(self):
        m = self.cache([1, 2, 3], [4, 5]).make_mask(N=2, return_array=True)
        assert m.shape == (2, 5) and m[0, 3] and not m[0, 4] and m[1, 4]

    def test_offset(self):
        assert self.cache([1, 2, 3, 4, 5], [6]).offset == 5


# ---- device pool -------------------------------------------------------------------

def _kv(rng, H, S, D):
    from sglang_mlx_b200.device_array import DeviceArray

    k = rng.standard_normal((1, H, S, D), dtype=np.float32)
    v = rng.standard_normal((1, H, S, D), dtype=np.float32)
    return k, v, DeviceArray.from_numpy(k), DeviceArray.from_numpy(v)


@pytest.mark.gpu
class TestMHATokenPool:
    """test_memory_pool.py:85-188 (fp32 pool, atol 1e-6 there; exact here)."""

    def pool(self, gpu):
        return MHATokenPool(pool_size=32, num_layers=2, n_kv_heads=4, head_dim=8, dtype="float32")

    def test_store_fetch_roundtrip(self, gpu):
        rng = np.random.default_rng(0)
        p = self.pool(gpu)
        k, v, kd, vd = _kv(rng, 4, 5, 8)
        p.store(0, [1, 2, 3, 4, 5], kd, vd)
        ko, vo = p.fetch(0, [1, 2, 3, 4, 5])
        assert ko.shape == k.shape
        np.testing.assert_array_equal(ko.to_numpy(), k)
        np.testing.assert_array_equal(vo.to_numpy(), v)

    def test_cross_layer_independence(self, gpu):
        rng = np.random.default_rng(1)
        p = self.pool(gpu)
        k0, _, k0d, v0d = _kv(rng, 4, 3, 8)
        k1, _, k1d, v1d = _kv(rng, 4, 3, 8)
        p.store(0, [1, 2, 3], k0d, v0d)
        p.store(1, [1, 2, 3], k1d, v1d)
        np.testing.assert_array_equal(p.fetch(0, [1, 2, 3])[0].to_numpy(), k0)
        np.testing.assert_array_equal(p.fetch(1, [1, 2, 3])[0].to_numpy(), k1)

    def test_non_contiguous_indices(self, gpu):
        rng = np.random.default_rng(2)
        p = self.pool(gpu)
        k, _, kd, vd = _kv(rng, 4, 3, 8)
        p.store(0, [5, 10, 20], kd, vd)
        np.testing.assert_array_equal(p.fetch(0, [5, 10, 20])[0].to_numpy(), k)

    def test_overwrite_existing_slot(self, gpu):
        rng = np.random.default_rng(3)
        p = self.pool(gpu)
        _, _, k1d, v1d = _kv(rng, 4, 1, 8)
        k2, _, k2d, v2d = _kv(rng, 4, 1, 8)
        p.store(0, [1], k1d, v1d)
        p.store(0, [1], k2d, v2d)
        np.testing.assert_array_equal(p.fetch(0, [1])[0].to_numpy(), k2)

    def test_fetch_subset_of_stored(self, gpu):
        rng = np.random.default_rng(4)
        p = self.pool(gpu)
        k, _, kd, vd = _kv(rng, 4, 5, 8)
        p.store(0, [1, 2, 3, 4, 5], kd, vd)
        ko, _ = p.fetch(0, [1, 2, 3])
        assert ko.shape == (1, 4, 3, 8)
        np.testing.assert_array_equal(ko.to_numpy(), k[:, :, :3, :])

    def test_matches_reference_pool(self, gpu, golden):
        """The reference MHATokenPool's scripted store/fetch results, bit for bit."""
        from sglang_mlx_b200.device_array import DeviceArray

        p = MHATokenPool(pool_size=40, num_layers=2, n_kv_heads=4, head_dim=8, dtype="float32")
        i = 0
        while f"pool/write{i}/layer" in golden:
            p.store(int(golden[f"pool/write{i}/layer"]), [int(x) for x in golden[f"pool/write{i}/idx"]],
                    DeviceArray.from_numpy(golden[f"pool/write{i}/k"]),
                    DeviceArray.from_numpy(golden[f"pool/write{i}/v"]))
            i += 1
        for layer in (0, 1):
            ko, vo = p.fetch(layer, [int(x) for x in golden["pool/fetch_idx"]])
            np.testing.assert_array_equal(ko.to_numpy(), golden[f"pool/fetch{layer}/k"])
            np.testing.assert_array_equal(vo.to_numpy(), golden[f"pool/fetch{layer}/v"])

    @pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
    def test_half_pools_and_torch_inputs(self, gpu, dtype):
        torch = pytest.importorskip("torch")
        rng = np.random.default_rng(5)
        p = MHATokenPool(pool_size=300, num_layers=1, n_kv_heads=8, head_dim=128, dtype=dtype)
        tdt = torch.float16 if dtype == "float16" else torch.bfloat16
        k = torch.from_numpy(rng.standard_normal((1, 8, 37, 128), dtype=np.float32)).to("cuda", tdt)
        v = torch.from_numpy(rng.standard_normal((1, 8, 37, 128), dtype=np.float32)).to("cuda", tdt)
        idx = list(rng.permutation(300)[:37] + 1)
        p.store(0, idx, k, v)
        ko, vo = p.fetch(0, idx)
        torch.cuda.synchronize()
        assert torch.equal(torch.from_dlpack(ko), k) and torch.equal(torch.from_dlpack(vo), v)


@pytest.mark.gpu
class TestPooledKVCache:
    """test_memory_pool.py:194-363 (store/fetch behaviour through the adapter)."""

    def pool(self):
        return MHATokenPool(pool_size=64, num_layers=2, n_kv_heads=4, head_dim=8, dtype="float32")

    def test_cold_start_prefill(self, gpu):
        rng = np.random.default_rng(10)
        cache = PooledKVCache(self.pool(), layer_idx=0)
        cache.set_indices(prefix_indices=[], new_indices=[1, 2, 3, 4, 5])
        assert cache.offset == 0
        k, _, kd, vd = _kv(rng, 4, 5, 8)
        ko, _ = cache.update_and_fetch(kd, vd)
        assert ko.shape == (1, 4, 5, 8)
        np.testing.assert_array_equal(ko.to_numpy(), k)

    def test_decode_with_prefix(self, gpu):
        rng = np.random.default_rng(11)
        pool = self.pool()
        cache = PooledKVCache(pool, layer_idx=0)
        kp, _, kpd, vpd = _kv(rng, 4, 5, 8)
        pool.store(0, [1, 2, 3, 4, 5], kpd, vpd)
        cache.set_indices(prefix_indices=[1, 2, 3, 4, 5], new_indices=[6])
        assert cache.offset == 5
        kn, _, knd, vnd = _kv(rng, 4, 1, 8)
        ko, _ = cache.update_and_fetch(knd, vnd)
        assert ko.shape == (1, 4, 6, 8)
        out = ko.to_numpy()
        np.testing.assert_array_equal(out[:, :, :5], kp)
        np.testing.assert_array_equal(out[:, :, 5:], kn)

    def test_state_property(self, gpu):
        rng = np.random.default_rng(12)
        cache = PooledKVCache(self.pool(), layer_idx=0)
        cache.set_indices(prefix_indices=[], new_indices=[1, 2, 3])
        _, _, kd, vd = _kv(rng, 4, 3, 8)
        cache.update_and_fetch(kd, vd)
        ks, vs = cache.state
        assert ks.shape == (1, 4, 3, 8)

    def test_state_empty_returns_none(self, gpu):
        cache = PooledKVCache(self.pool(), layer_idx=0)
        cache.set_indices(prefix_indices=[], new_indices=[])
        assert cache.state == (None, None)

    def test_prefill_then_decode_end_to_end(self, gpu):
        """test_memory_pool.py:451-538 (allocator + pool + adapter)."""
        rng = np.random.default_rng(13)
        alloc = TokenPoolAllocator(32)
        pool = MHATokenPool(32, 2, 2, 4, dtype="float32")
        slots = alloc.alloc(4)
        caches = [PooledKVCache(pool, i) for i in range(2)]
        k_in, _, kd, vd = _kv(rng, 2, 4, 4)
        for c in caches:
            c.set_indices(prefix_indices=[], new_indices=slots)
            assert c.update_and_fetch(kd, vd)[0].shape == (1, 2, 4, 4)
        new_slot = alloc.alloc(1)
        _, _, knd, vnd = _kv(rng, 2, 1, 4)
        for c in caches:
            c.set_indices(prefix_indices=slots, new_indices=new_slot)
            assert c.offset == 4
            ko, _ = c.update_and_fetch(knd, vnd)
            assert ko.shape == (1, 2, 5, 4)
            np.testing.assert_array_equal(ko.to_numpy()[:, :, :4], k_in)



class TestPagedAllocator:
    """page_size > 1: whole pages, page p = slots p*ps+1 .. (p+1)*ps."""

    def test_alloc_takes_whole_pages_in_order(self):
        a = TokenPoolAllocator(16, page_size=4)
        assert a.alloc(5) == [1, 2, 3, 4, 5]
        assert a.available_size == 8
        assert a.alloc(2) == [9, 10]

    def test_alloc_extend_fills_the_page_first(self):
        a = TokenPoolAllocator(16, page_size=4)
        s = a.alloc(3)
        other = a.alloc(1)
        assert other == [5]
        s += a.alloc_extend(s[-1], 3)
        assert s == [1, 2, 3, 4, 9, 10]
        assert a.alloc_extend(other[-1], 2) == [6, 7]

    def test_pages_return_when_every_slot_is_freed(self):
        a = TokenPoolAllocator(8, page_size=4)
        s = a.alloc(6)
        a.free(s[:3])
        assert a.available_size == 0
        a.free(s[3:4])
        assert a.available_size == 4
        a.free(s[4:])
        assert a.available_size == 8
        assert len(set(a.alloc(8))) == 8

    def test_overflow_and_bad_sizes(self):
        a = TokenPoolAllocator(8, page_size=4)
        a.alloc(5)
        with pytest.raises(MemoryError):
            a.alloc(1)
        with pytest.raises(ValueError):
            TokenPoolAllocator(10, page_size=4)
        a.clear()
        assert a.available_size == 8

    def test_page_size_one_is_the_reference_allocator(self):
        a, b = TokenPoolAllocator(10), TokenPoolAllocator(10, page_size=1)
        assert a.alloc(3) == b.alloc(3) == [3, 2, 1]
        assert b.alloc_extend(1, 2) == a.alloc(2)

    def test_slots_to_pages(self):
        from sglang_mlx_b200.srt.mem_cache.memory_pool import slots_to_pages

        assert list(slots_to_pages([1, 2, 3, 4, 9, 10], 4)) == [0, 2]
        assert slots_to_pages([1, 2, 4], 4) is None
        assert slots_to_pages([2, 3], 4) is None
        assert slots_to_pages([5, 6, 7, 8, 1], 4).tolist() == [1, 0]
        assert slots_to_pages([3, 2, 1], 1) is None
