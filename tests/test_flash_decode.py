"""GPU parity tests of the token-major decode (kvc_paged_attention_flash): the
reshape_and_cache_flash layout [nb, bs, H, D] and the MHATokenPool buffers
[slots, H, D] (block size 1, slot lists as block tables), through
metal_kernels.paged_attention_flash, MHATokenPool.decode and
PooledKVCache.update_and_attend.  Oracle: kv_oracle.paged_attention_flash
(float64), itself pinned to the golden-pinned paged_attention_v1
restatement in tests/test_oracle.py."""

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close, fill_cache, flash_case, upload_case, upload_flash
from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray
from sglang_mlx_b200.srt.mem_cache.memory_pool import MHATokenPool, PooledKVCache, TokenPoolAllocator

pytestmark = pytest.mark.gpu


def oracle_flash(fc, alibi=None, max_seq_len=None):
    c = fc["c"]
    fk = np.zeros(fc["shape"], np.float32)
    fv = np.zeros(fc["shape"], np.float32)
    kv_oracle.reshape_and_cache_flash(kv_oracle.round_to(c["k"], c["dtype"]), kv_oracle.round_to(c["v"], c["dtype"]),
                                      fk, fv, fc["slots"])
    return kv_oracle.paged_attention_flash(kv_oracle.round_to(c["q"], c["dtype"]), fk, fv, fc["tables"],
                                           c["context_lens"], c["num_kv_heads"], c["scale"],
                                           max_seq_len or c["max_seq_len"], alibi)


def run_flash(fc, d, partition_size=0, alibi=None, max_seq_len=None):
    c = fc["c"]
    return mk.paged_attention_flash(d["q"], d["kc"], d["vc"], d["tables"], d["lens"], c["num_kv_heads"], c["scale"],
                                    fc["bs"], max_seq_len or c["max_seq_len"], alibi,
                                    partition_size=partition_size).to_numpy()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [1, 8, 16, 32])
def test_layouts_dtypes_head_sizes(gpu, dtype, D, bs):
    fc = flash_case(4000 + D + bs, dtype, 3, 8, 2, D, bs, [1, 37, 300])
    d = upload_flash(fc)
    ref = oracle_flash(fc)
    assert_close(run_flash(fc, d), ref, ATOL_NS, RTOL_NS, f"{dtype} D{D} bs{bs}")
    assert_close(run_flash(fc, d, partition_size=64), ref, ATOL_NS, RTOL_NS, f"{dtype} D{D} bs{bs} split")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (16, 4), (28, 4), (32, 4), (32, 2), (16, 1), (64, 2)])
def test_group_sizes(gpu, Hq, Hkv):
    fc = flash_case(4100 + Hq + Hkv, "bfloat16", 3, Hq, Hkv, 128, 1, [200, 33, 1500])
    d = upload_flash(fc)
    if Hq // Hkv > 16:  # one tensor-core tile holds at most 16 query heads of a group
        with pytest.raises(NotImplementedError, match="16 query heads"):
            run_flash(fc, d)
        return
    assert_close(run_flash(fc, d), oracle_flash(fc), ATOL_NS, RTOL_NS, f"G={Hq // Hkv}")


def test_alibi_and_split(gpu):
    fc = flash_case(4200, "float16", 3, 8, 2, 128, 16, [17, 2000, 64])
    d = upload_flash(fc)
    slopes = (2.0 ** -np.arange(1, 9)).astype(np.float32)
    ref = oracle_flash(fc, alibi=slopes)
    al = DeviceArray.from_numpy(slopes)
    assert_close(run_flash(fc, d, alibi=al), ref, ATOL_NS, RTOL_NS, "alibi")
    assert_close(run_flash(fc, d, partition_size=256, alibi=al), ref, ATOL_NS, RTOL_NS, "alibi split")


def test_mixed_lengths_zero_rows_and_max_seq_len(gpu):
    lens = [0, 1, 15, 16, 17, 511, 512, 513, 1000, 0, 3000]
    fc = flash_case(4300, "bfloat16", len(lens), 16, 4, 128, 1, [max(x, 1) for x in lens])
    fc["c"]["context_lens"] = np.array(lens, np.int32)
    d = upload_flash(fc)
    for psize in (0, 256):
        out = run_flash(fc, d, partition_size=psize)
        assert not out[0].any() and not out[9].any()
        assert_close(out, oracle_flash(fc), ATOL_NS, RTOL_NS, f"mixed P={psize}")
    out = run_flash(fc, d, max_seq_len=1000)
    assert not out[10].any()
    assert_close(out, oracle_flash(fc, max_seq_len=1000), ATOL_NS, RTOL_NS, "max_seq_len")


def test_nan_in_unused_slots_never_leaks(gpu):
    fc = flash_case(4400, "float16", 2, 8, 2, 128, 1, [20, 40])
    d = upload_flash(fc)
    # poison every slot no sequence uses
    used = set(fc["slots"].tolist())
    kc = d["kc"].to_numpy()
    vc = d["vc"].to_numpy()
    unused = np.array([i for i in range(kc.shape[0]) if i not in used])
    kc[unused] = np.nan
    vc[unused] = np.nan
    d["kc"] = DeviceArray.from_numpy(kc)
    d["vc"] = DeviceArray.from_numpy(vc)
    out = run_flash(fc, d)
    assert np.isfinite(out).all()
    assert_close(out, oracle_flash(fc), ATOL_NS, RTOL_NS, "nan neighbours")


def test_out_of_range_slot_is_skipped_and_flagged(gpu):
    fc = flash_case(4500, "float16", 2, 8, 2, 128, 1, [40, 40])
    d = upload_flash(fc)
    t = fc["tables"].copy()
    t[1, 5] = 10_000_000
    d["tables"] = DeviceArray.from_numpy(t)
    gpu.get_status(clear=True)
    out = run_flash(fc, d)
    assert np.isfinite(out).all()
    assert gpu.get_status(clear=True) & _lib.STATUS_BLOCK_OOB


def test_unsupported_dtype_is_refused(gpu):
    fc = flash_case(4600, "float32", 2, 8, 2, 128, 1, [4, 5])
    d = upload_flash(fc)
    with pytest.raises(NotImplementedError, match="float16/bfloat16"):
        run_flash(fc, d)


def test_matches_paged_layout_at_scale(gpu):
    """Config 2's shape (32 sequences here, U[512, 4096] tokens, 32/8 heads, bf16):
    the same tokens through the vLLM layout (paged_attention_v1) and the token pool."""
    rng = np.random.default_rng(2024)
    lens = rng.integers(512, 4097, size=32)
    fc = flash_case(4700, "bfloat16", 32, 32, 8, 128, 1, lens)
    d = upload_flash(fc)
    c = fc["c"]
    pd = upload_case(c)
    fill_cache(pd)
    v1 = mk.paged_attention_v1(pd["q"], pd["k_cache"], pd["v_cache"], pd["block_tables"], pd["context_lens"], 8,
                               c["scale"], 16, c["max_seq_len"]).to_numpy()
    for psize in (0, 1024):
        assert_close(run_flash(fc, d, partition_size=psize), v1.astype(np.float64), ATOL_NS, RTOL_NS,
                     f"pool vs paged P={psize}")


# ---- the pool API ----------------------------------------------------------------

def _pool_batch(seed, dtype, hq, hkv, d, prompt_lens, pool_size=6000, page_size=1):
    rng = np.random.default_rng(seed)
    pool = MHATokenPool(pool_size, 2, hkv, d, dtype, page_size=page_size)
    alloc = TokenPoolAllocator(pool_size, page_size=page_size)
    slots, keys = [], []
    for n in prompt_lens:
        idx = alloc.alloc(int(n))
        kv = [kv_oracle.round_to(rng.standard_normal((1, hkv, n, d)).astype(np.float32), dtype) for _ in range(2)]
        for layer in range(2):
            pool.store(layer, idx, DeviceArray.from_numpy(kv[0], dtype=dtype), DeviceArray.from_numpy(kv[1],
                                                                                                      dtype=dtype))
        slots.append(idx)
        keys.append(kv)
    return pool, alloc, slots, keys, rng


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_pool_decode_matches_oracle(gpu, dtype):
    prompt_lens = [1, 17, 300, 1234]
    pool, _, slots, keys, rng = _pool_batch(4800, dtype, 32, 8, 128, prompt_lens)
    B, T = len(prompt_lens), max(prompt_lens)
    tables = np.zeros((B, T), np.int32)
    for b, idx in enumerate(slots):
        tables[b, :len(idx)] = idx
    q = kv_oracle.round_to(rng.standard_normal((B, 32, 128)).astype(np.float32), dtype)
    out = pool.decode(1, DeviceArray.from_numpy(q, dtype=dtype), tables, np.array(prompt_lens, np.int32)).to_numpy()
    ref = np.zeros((B, 32, 128))
    for b in range(B):
        k = keys[b][0][0].transpose(1, 0, 2)  # (S, H, D)
        v = keys[b][1][0].transpose(1, 0, 2)
        for h in range(8):
            ref[b, 4 * h:4 * h + 4] = kv_oracle.attend(q[b, 4 * h:4 * h + 4], k[:, h], v[:, h], 128 ** -0.5)
    assert_close(out, ref, ATOL_NS, RTOL_NS, f"pool decode {dtype}")


def test_pooled_cache_update_and_attend_equals_gather_path(gpu):
    """update_and_attend (append + decode on the pool) against update_and_fetch
    (append + gather) followed by the oracle's attention, over several steps."""
    dtype = "bfloat16"
    pool, alloc, slots, keys, rng = _pool_batch(4900, dtype, 16, 4, 128, [700])
    prefix = list(slots[0])
    for step in range(3):
        new = alloc.alloc(1)
        caches = [PooledKVCache(pool, 0), PooledKVCache(pool, 1)]
        q = kv_oracle.round_to(rng.standard_normal((1, 16, 1, 128)).astype(np.float32), dtype)
        kn = kv_oracle.round_to(rng.standard_normal((1, 4, 1, 128)).astype(np.float32), dtype)
        vn = kv_oracle.round_to(rng.standard_normal((1, 4, 1, 128)).astype(np.float32), dtype)
        caches[0].set_indices(prefix, new)
        caches[1].set_indices(prefix, new)
        out = caches[0].update_and_attend(DeviceArray.from_numpy(q, dtype=dtype), DeviceArray.from_numpy(kn, dtype=dtype),
                                          DeviceArray.from_numpy(vn, dtype=dtype))
        assert out.shape == (1, 16, 1, 128)
        kf, vf = caches[1].update_and_fetch(DeviceArray.from_numpy(kn, dtype=dtype),
                                            DeviceArray.from_numpy(vn, dtype=dtype))
        kf, vf = kf.to_numpy()[0], vf.to_numpy()[0]  # (H, T, D)
        ref = np.stack([kv_oracle.attend(q[0, 4 * h:4 * h + 4, 0], kf[h], vf[h], 128 ** -0.5) for h in range(4)])
        assert_close(out.to_numpy()[0, :, 0], ref.reshape(16, 128), ATOL_NS, RTOL_NS, f"step {step}")
        prefix = prefix + new
    with pytest.raises(ValueError, match="same N"):
        caches[0].update_and_attend(DeviceArray.from_numpy(np.zeros((1, 16, 2, 128), np.float32), dtype=dtype),
                                    DeviceArray.from_numpy(np.zeros((1, 4, 3, 128), np.float32), dtype=dtype),
                                    DeviceArray.from_numpy(np.zeros((1, 4, 3, 128), np.float32), dtype=dtype))


# ---- blocks of consecutive token rows: tensor copies (kFlashTma) ---------------------

@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [16, 32, 64])
def test_tensor_copy_rows_match_row_copies(gpu, dtype, D, bs, monkeypatch):
    """Block sizes that are multiples of 16 read each 16-token group of a head with
    tensor copies; KVC_FLASH_COPY=cpasync forces the per-lane 16-byte row copies.
    Both agree with the oracle, single pass and split-K."""
    fc = flash_case(5000 + D + bs, dtype, 4, 8, 2, D, bs, [1, 16, 333, 2000])
    d = upload_flash(fc)
    ref = oracle_flash(fc)
    for psize in (0, 256):
        tma = run_flash(fc, d, partition_size=psize)
        monkeypatch.setenv("KVC_FLASH_COPY", "cpasync")
        rows = run_flash(fc, d, partition_size=psize)
        monkeypatch.delenv("KVC_FLASH_COPY")
        assert_close(tma, ref, ATOL_NS, RTOL_NS, f"tensor copies bs{bs} P={psize}")
        assert_close(rows, ref, ATOL_NS, RTOL_NS, f"row copies bs{bs} P={psize}")
    assert gpu.get_status(clear=True) == 0


# ---- dense token rows in any order (slot lists): 4-row tensor gathers (kFlashGather) --------

def scatter_slots(fc, seed):
    """A token-pool case (block size 1) with its slots moved to a random
    permutation of the pool (slot 0, the padding slot, stays): neighbouring
    tokens of a sequence land anywhere."""
    rng = np.random.default_rng(seed)
    n = fc["shape"][0]
    perm = np.concatenate([[0], 1 + rng.permutation(n - 1)]).astype(np.int64)
    fc = dict(fc)
    fc["slots"] = perm[fc["slots"].astype(np.int64)].astype(np.int32)
    fc["tables"] = perm[fc["tables"].astype(np.int64)].astype(np.int32)
    return fc


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [1, 8])
def test_gathered_rows_match_row_copies(gpu, dtype, D, bs, monkeypatch):
    """KVC_FLASH_COPY=gather reads each token's K and V rows of slot lists
    (block size 1) and of 8-token blocks by 4-row tensor gathers; the default
    is the per-lane 16-byte row copies.  Lengths end inside a 4-row quad and
    inside a 16-token group; both forms agree with the oracle, single pass and
    split-K."""
    fc = flash_case(5100 + D + bs, dtype, 5, 8, 2, D, bs, [1, 3, 17, 334, 2001])
    if bs == 1:
        fc = scatter_slots(fc, 5100 + D)
    d = upload_flash(fc)
    ref = oracle_flash(fc)
    for psize in (0, 256):
        monkeypatch.setenv("KVC_FLASH_COPY", "gather")
        gat = run_flash(fc, d, partition_size=psize)
        monkeypatch.delenv("KVC_FLASH_COPY")
        rows = run_flash(fc, d, partition_size=psize)
        assert_close(gat, ref, ATOL_NS, RTOL_NS, f"gathers bs{bs} P={psize}")
        assert_close(rows, ref, ATOL_NS, RTOL_NS, f"row copies bs{bs} P={psize}")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("copy", ["gather", "cpasync"])
def test_gathered_rows_bad_slots_inside_a_group(gpu, copy, monkeypatch):
    """Out-of-range slots in the middle of a 16-token group (and one as its first
    token) are flagged and masked; the other tokens of the group still count:
    the result equals the oracle over the same table with those tokens dropped
    (tensor gathers and row copies alike)."""
    fc = scatter_slots(flash_case(5200, "bfloat16", 2, 8, 2, 128, 1, [48, 48]), 5200)
    d = upload_flash(fc)
    t = fc["tables"].copy()
    bad = [(0, 16), (0, 21), (1, 5)]
    for b, i in bad:
        t[b, i] = 10_000_000
    d["tables"] = DeviceArray.from_numpy(t)
    gpu.get_status(clear=True)
    monkeypatch.setenv("KVC_FLASH_COPY", copy)
    out = run_flash(fc, d)
    monkeypatch.delenv("KVC_FLASH_COPY")
    assert gpu.get_status(clear=True) & _lib.STATUS_BLOCK_OOB
    # the oracle without those tokens: their keys get a score of -inf
    c = fc["c"]
    fk = np.zeros(fc["shape"], np.float32)
    fv = np.zeros(fc["shape"], np.float32)
    kv_oracle.reshape_and_cache_flash(kv_oracle.round_to(c["k"], c["dtype"]), kv_oracle.round_to(c["v"], c["dtype"]),
                                      fk, fv, fc["slots"])
    q = kv_oracle.round_to(c["q"], c["dtype"]).astype(np.float64)
    ref = np.zeros_like(q)
    G = 8 // 2
    for b in range(2):
        n = int(c["context_lens"][b])
        keep = [i for i in range(n) if (b, i) not in bad]
        slots = fc["tables"][b, keep]
        for h in range(8):
            k = fk[slots, h // G].astype(np.float64)
            v = fv[slots, h // G].astype(np.float64)
            sc = k @ q[b, h] * c["scale"]
            w = np.exp(sc - sc.max())
            ref[b, h] = w @ v / w.sum()
    assert_close(out, ref, ATOL_NS, RTOL_NS, "bad slots masked")


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_paged_pool_decode_pages_matches_slot_lists(gpu, dtype):
    """A pool whose allocator hands out 16-token pages: requests allocated in
    turns (alloc, then alloc_extend token by token) hold interleaved pages;
    decode_pages over the page tables equals decode over the slot lists and the
    oracle."""
    ps = 16
    rng = np.random.default_rng(5100)
    pool = MHATokenPool(4096, 2, 4, 128, dtype, page_size=ps)
    alloc = TokenPoolAllocator(4096, page_size=ps)
    lens = [5, 40, 300, 17]
    slots = [alloc.alloc(1) for _ in lens]
    for step in range(1, max(lens)):
        for b, n in enumerate(lens):
            if step < n:
                slots[b] += alloc.alloc_extend(slots[b][-1], 1)
    keys = []
    for b, n in enumerate(lens):
        kv = [kv_oracle.round_to(rng.standard_normal((1, 4, n, 128)).astype(np.float32), dtype) for _ in range(2)]
        pool.store(1, slots[b], DeviceArray.from_numpy(kv[0], dtype=dtype), DeviceArray.from_numpy(kv[1], dtype=dtype))
        keys.append(kv)
    from sglang_mlx_b200.srt.mem_cache.memory_pool import slots_to_pages

    T = max(lens)
    st = np.zeros((len(lens), T), np.int32)
    pt = np.zeros((len(lens), -(-T // ps)), np.int32)
    for b, idx in enumerate(slots):
        st[b, :len(idx)] = idx
        pages = slots_to_pages(idx, ps)
        assert pages is not None
        pt[b, :len(pages)] = pages
    q = kv_oracle.round_to(rng.standard_normal((len(lens), 16, 128)).astype(np.float32), dtype)
    qd = DeviceArray.from_numpy(q, dtype=dtype)
    by_pages = pool.decode_pages(1, qd, pt, np.array(lens, np.int32)).to_numpy()
    by_slots = pool.decode(1, qd, st, np.array(lens, np.int32)).to_numpy()
    ref = np.zeros((len(lens), 16, 128))
    for b in range(len(lens)):
        k = keys[b][0][0].transpose(1, 0, 2)
        v = keys[b][1][0].transpose(1, 0, 2)
        for h in range(4):
            ref[b, 4 * h:4 * h + 4] = kv_oracle.attend(q[b, 4 * h:4 * h + 4], k[:, h], v[:, h], 128 ** -0.5)
    assert_close(by_pages, ref, ATOL_NS, RTOL_NS, "decode_pages")
    assert_close(by_slots, ref, ATOL_NS, RTOL_NS, "decode (slot lists)")
    assert gpu.get_status(clear=True) == 0


def test_paged_pool_update_and_attend_equals_gather_path(gpu):
    """update_and_attend on a page-granular pool reads the request's pages (its
    slots fill them in order) and matches update_and_fetch + the oracle."""
    dtype = "bfloat16"
    pool, alloc, slots, keys, rng = _pool_batch(5200, dtype, 16, 4, 128, [700], pool_size=4096, page_size=32)
    prefix = list(slots[0])
    for step in range(3):
        new = alloc.alloc_extend(prefix[-1], 1)
        caches = [PooledKVCache(pool, 0), PooledKVCache(pool, 1)]
        q = kv_oracle.round_to(rng.standard_normal((1, 16, 1, 128)).astype(np.float32), dtype)
        kn = kv_oracle.round_to(rng.standard_normal((1, 4, 1, 128)).astype(np.float32), dtype)
        vn = kv_oracle.round_to(rng.standard_normal((1, 4, 1, 128)).astype(np.float32), dtype)
        caches[0].set_indices(prefix, new)
        caches[1].set_indices(prefix, new)
        out = caches[0].update_and_attend(DeviceArray.from_numpy(q, dtype=dtype), DeviceArray.from_numpy(kn, dtype=dtype),
                                          DeviceArray.from_numpy(vn, dtype=dtype))
        kf, vf = caches[1].update_and_fetch(DeviceArray.from_numpy(kn, dtype=dtype),
                                            DeviceArray.from_numpy(vn, dtype=dtype))
        kf, vf = kf.to_numpy()[0], vf.to_numpy()[0]
        ref = np.stack([kv_oracle.attend(q[0, 4 * h:4 * h + 4, 0], kf[h], vf[h], 128 ** -0.5) for h in range(4)])
        assert_close(out.to_numpy()[0, :, 0], ref.reshape(16, 128), ATOL_NS, RTOL_NS, f"step {step}")
        prefix = prefix + new
    assert gpu.get_status(clear=True) == 0
