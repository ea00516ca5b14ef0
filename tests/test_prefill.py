"""GPU parity tests of paged prefill / extend attention (kvc_paged_prefill,
metal_kernels.paged_prefill_attention, PooledKVCache.update_and_attend with
N > 1).  Oracle: kv_oracle.paged_prefill (float64 SDPA over the gathered K/V
under the offset-causal / window mask of PooledKVCache.make_mask), whose mask
is pinned to the reference's make_mask tests and whose SDPA is cross-checked
against torch in tests/test_oracle.py.  Cases: every layout (paged block sizes
8/16/32, flash layout, token pool), dtypes, head sizes, group sizes, sliding
windows, ragged batches with empty and single-token sequences, a long chunk on
a long prefix, device-side index errors, and the pool wiring."""

import math

import numpy as np
import pytest

import cases
from helpers import (ATOL_NS, RTOL_NS, assert_close, fill_cache, flash_case, oracle_fill, oracle_flash_caches,
                     upload_case, upload_flash)
from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray
from sglang_mlx_b200.srt.mem_cache.memory_pool import MHATokenPool, PooledKVCache, TokenPoolAllocator

pytestmark = pytest.mark.gpu


def prefill_case(seed, dtype, hq, hkv, d, layout, bs, prefixes, qlens):
    """Sequences b with prefixes[b] cached tokens and qlens[b] new ones (whose K/V
    are in the cache too).  layout "paged" (vLLM layout, block size bs) or
    "flash" (token-major, block size bs; bs 1 = the token pool)."""
    B = len(prefixes)
    kvl = np.asarray([p + q for p, q in zip(prefixes, qlens)], np.int32)
    rng = np.random.default_rng(seed + 99)
    q = cases.cast(rng.standard_normal((int(sum(qlens)), hq, d), dtype=np.float32), dtype)
    indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    if layout == "paged":
        c = cases.paged_batch(seed, dtype, B, hq, hkv, d, bs, kvl)
        dev = upload_case(c)
        fill_cache(dev)
        kc, vc = oracle_fill(c, dtype)
        tables, kcd, vcd = c["block_tables"], dev["k_cache"], dev["v_cache"]
    else:
        fc = flash_case(seed, dtype, B, hq, hkv, d, bs, kvl)
        dev = upload_flash(fc)
        kc, vc = oracle_flash_caches(fc)
        tables, kcd, vcd = fc["tables"], dev["kc"], dev["vc"]
    return dict(q=q, qd=DeviceArray.from_numpy(q, dtype=dtype), kc=kc, vc=vc, kcd=kcd, vcd=vcd, tables=tables,
                indptr=indptr, kvl=kvl, hkv=hkv, scale=1.0 / math.sqrt(d), bs=bs, dtype=dtype)


def run(c, window=None, indptr=None, kvl=None, max_q_len=None):
    return mk.paged_prefill_attention(c["qd"], c["kcd"], c["vcd"], DeviceArray.from_numpy(c["tables"]),
                                      c["indptr"] if indptr is None else indptr,
                                      DeviceArray.from_numpy(c["kvl"] if kvl is None else kvl), c["hkv"], c["scale"],
                                      c["bs"], window_size=window, max_q_len=max_q_len).to_numpy()


def ref(c, window=None):
    return kv_oracle.paged_prefill(kv_oracle.round_to(c["q"], c["dtype"]), c["kc"], c["vc"], c["tables"], c["indptr"],
                                   c["kvl"], c["hkv"], c["scale"], window)


LAYOUTS = [("paged", 8), ("paged", 16), ("paged", 32), ("flash", 16), ("flash", 1)]


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("layout,bs", LAYOUTS)
def test_layouts_dtypes_head_sizes(gpu, dtype, D, layout, bs):
    c = prefill_case(6000 + D + bs, dtype, 16, 4, D, layout, bs, [0, 100, 300, 37], [37, 64, 1, 130])
    assert_close(run(c), ref(c), ATOL_NS, RTOL_NS, f"{layout} bs{bs} {dtype} D{D}")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (6, 2), (28, 4), (32, 8), (64, 8), (32, 1)])
def test_group_sizes(gpu, Hq, Hkv):
    c = prefill_case(6100 + Hq + Hkv, "bfloat16", Hq, Hkv, 128, "flash", 1, [50, 0, 211], [70, 33, 5])
    assert_close(run(c), ref(c), ATOL_NS, RTOL_NS, f"G={Hq // Hkv}")


@pytest.mark.parametrize("window", [1, 5, 64, 333, 100000])
@pytest.mark.parametrize("layout,bs", [("paged", 16), ("flash", 1)])
def test_sliding_windows(gpu, window, layout, bs):
    c = prefill_case(6200 + window, "bfloat16", 16, 4, 128, layout, bs, [0, 400, 90], [200, 96, 1])
    assert_close(run(c, window=window), ref(c, window=window), ATOL_NS, RTOL_NS, f"window {window}")


def test_long_chunk_on_long_prefix(gpu):
    """A 512-token chunk on a 3000-token prefix and a 1024-token prompt, with
    the heads and block size of BASELINE config 5 (28/4, bs 32, bf16)."""
    c = prefill_case(6300, "bfloat16", 28, 4, 128, "paged", 32, [3000, 0], [512, 1024])
    assert_close(run(c), ref(c), ATOL_NS, RTOL_NS, "long chunk")
    assert gpu.get_status(clear=True) == 0


def test_single_new_token_equals_decode(gpu):
    """One new token per sequence is a decode step: the result matches
    paged_attention_v1 on the same cache."""
    c = prefill_case(6400, "float16", 32, 8, 128, "paged", 16, [0, 15, 16, 999], [1, 1, 1, 1])
    out = run(c)
    dec = mk.paged_attention_v1(c["qd"], c["kcd"], c["vcd"], DeviceArray.from_numpy(c["tables"]),
                                DeviceArray.from_numpy(c["kvl"]), 8, c["scale"], 16,
                                c["tables"].shape[1] * 16).to_numpy()
    assert_close(out, dec.astype(np.float64), ATOL_NS, RTOL_NS, "prefill vs decode")
    assert_close(out, ref(c), ATOL_NS, RTOL_NS, "oracle")


def test_empty_sequences_and_whole_prompts(gpu):
    """Sequences with no new tokens leave no rows; a prompt with no prefix is
    plain causal attention."""
    c = prefill_case(6500, "bfloat16", 16, 4, 128, "paged", 16, [10, 0, 64, 0], [0, 77, 0, 3])
    assert_close(run(c), ref(c), ATOL_NS, RTOL_NS, "ragged")
    causal = kv_oracle.offset_causal_mask(77, 77)
    assert causal[5, 5] and not causal[5, 6]


def test_device_indptr_and_default_grid(gpu):
    """qo_indptr on the device: max_q_len defaults to num_tokens (extra row
    tiles exit at once); an explicit max_q_len gives the same rows."""
    c = prefill_case(6600, "float16", 16, 4, 128, "flash", 16, [5, 200], [40, 9])
    dind = DeviceArray.from_numpy(c["indptr"])
    r = ref(c)
    assert_close(run(c, indptr=dind), r, ATOL_NS, RTOL_NS, "default max_q_len")
    assert_close(run(c, indptr=dind, max_q_len=40), r, ATOL_NS, RTOL_NS, "max_q_len 40")


def test_bad_kv_lens_are_flagged(gpu):
    """kv_lens below a sequence's new-token count (or past its table) is an
    index error the host cannot see: the status word says so and the rows are 0."""
    c = prefill_case(6700, "float16", 16, 4, 128, "paged", 16, [20, 30], [8, 8])
    gpu.get_status(clear=True)
    out = run(c, kvl=np.asarray([5, 38], np.int32))
    assert gpu.get_status(clear=True) & _lib.STATUS_INDEX_OOB
    assert not out[:8].any()
    good = ref(c)[8:]
    assert_close(out[8:], good, ATOL_NS, RTOL_NS, "the valid sequence")
    run(c, kvl=np.asarray([28, 10 ** 6], np.int32))
    assert gpu.get_status(clear=True) & _lib.STATUS_INDEX_OOB


def test_invalid_and_unsupported_arguments(gpu):
    c = prefill_case(6800, "float16", 16, 4, 128, "paged", 16, [3], [4])
    with pytest.raises(ValueError, match="qo_indptr"):
        mk.paged_prefill_attention(c["qd"], c["kcd"], c["vcd"], c["tables"], np.array([0], np.int32), c["kvl"], 4,
                                   c["scale"], 16)
    with pytest.raises(ValueError, match="num_kv_heads"):
        mk.paged_prefill_attention(c["qd"], c["kcd"], c["vcd"], c["tables"], c["indptr"], c["kvl"], 3, c["scale"], 16)
    q32 = DeviceArray.from_numpy(c["q"].astype(np.float32))
    with pytest.raises(NotImplementedError, match="float16/bfloat16"):
        mk.paged_prefill_attention(q32, c["kcd"], c["vcd"], c["tables"], c["indptr"], c["kvl"], 4, c["scale"], 16)


@pytest.mark.parametrize("window", [None, 48])
def test_pooled_cache_prefill_equals_gather_path(gpu, window):
    """PooledKVCache.update_and_attend with N > 1 (append + prefill on the pool)
    against update_and_fetch (append + gather) and the oracle's masked SDPA,
    for a chunk on a cached prefix and then a whole prompt."""
    dtype = "bfloat16"
    rng = np.random.default_rng(6900)
    pool = MHATokenPool(4000, 2, 4, 128, dtype)
    alloc = TokenPoolAllocator(4000)
    prefix = []
    for n in (300, 120):  # first chunk on no prefix, second on the first's slots
        new = alloc.alloc(n)
        caches = [PooledKVCache(pool, 0), PooledKVCache(pool, 1)]
        for cc in caches:
            cc.set_indices(prefix, new)
        q = kv_oracle.round_to(rng.standard_normal((1, 16, n, 128)).astype(np.float32), dtype)
        kn = kv_oracle.round_to(rng.standard_normal((1, 4, n, 128)).astype(np.float32), dtype)
        vn = kv_oracle.round_to(rng.standard_normal((1, 4, n, 128)).astype(np.float32), dtype)
        up = lambda a: DeviceArray.from_numpy(a, dtype=dtype)  # noqa: E731
        out = caches[0].update_and_attend(up(q), up(kn), up(vn), window_size=window)
        assert out.shape == (1, 16, n, 128)
        kf, vf = caches[1].update_and_fetch(up(kn), up(vn))
        kf, vf = kf.to_numpy()[0], vf.to_numpy()[0]  # (H, T, D)
        T = kf.shape[1]
        mask = kv_oracle.offset_causal_mask(n, T, window)
        r = np.stack([kv_oracle.sdpa_masked(q[0, h], kf[h // 4], vf[h // 4], 128 ** -0.5, mask) for h in range(16)])
        assert_close(out.to_numpy()[0], r, ATOL_NS, RTOL_NS, f"chunk of {n} on {len(prefix)}")
        prefix = prefix + list(new)


def test_non_dense_key_cache_pages(gpu):
    """A key cache that is a view with a wider block stride (every page still
    dense) takes the per-page path of the tcgen05 kernel (no row gathers)."""
    c = prefill_case(7000, "bfloat16", 16, 4, 128, "paged", 32, [300, 0], [200, 77])
    kc = c["kcd"].to_numpy()
    nb, H = kc.shape[0], kc.shape[1]
    wide = np.zeros((nb, H + 1) + kc.shape[2:], np.float32)
    wide[:, :H] = kc
    wd = DeviceArray.from_numpy(wide, dtype="bfloat16")
    view = wd[:, :H]
    out = mk.paged_prefill_attention(c["qd"], view, c["vcd"], DeviceArray.from_numpy(c["tables"]), c["indptr"],
                                     DeviceArray.from_numpy(c["kvl"]), 4, c["scale"], 32).to_numpy()
    assert_close(out, ref(c), ATOL_NS, RTOL_NS, "non-dense K")
    assert gpu.get_status(clear=True) == 0



@pytest.fixture
def one_tile_form(monkeypatch):
    """Forces the two-tile tcgen05 kernel for the test (KVC_PREFILL_PAIR=1, read
    at every launch; unset, it runs only when its items fill the SMs) and
    returns a runner of a callable on the one-tile kernel (KVC_PREFILL_PAIR=0)."""
    monkeypatch.setenv("KVC_PREFILL_PAIR", "1")

    def call(fn):
        monkeypatch.setenv("KVC_PREFILL_PAIR", "0")
        try:
            return fn()
        finally:
            monkeypatch.setenv("KVC_PREFILL_PAIR", "1")
    return call


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D,bs", [(64, 16), (128, 16), (64, 32), (128, 32)])
def test_two_tile_and_one_tile_forms(gpu, one_tile_form, dtype, D, bs):
    """The gathered-K tcgen05 kernel runs items of two 128-row tiles: rows of
    tile B past the sequence (B empty), odd tile counts (3 and 5 tiles of G x
    new tokens), a one-row tile and a whole pair all match the oracle and the
    one-tile kernel."""
    # G = 4: 96 new tokens = 3 tiles, 160 = 5 tiles, 32 = 1 tile, 64 = 2 tiles, 1 token = 4 rows
    c = prefill_case(7100 + D + bs, dtype, 16, 4, D, "paged", bs, [0, 500, 33, 128, 7], [96, 160, 32, 64, 1])
    r = ref(c)
    two = run(c)
    assert_close(two, r, ATOL_NS, RTOL_NS, f"two-tile {dtype} D{D} bs{bs}")
    one = one_tile_form(lambda: run(c))
    assert_close(one, r, ATOL_NS, RTOL_NS, f"one-tile {dtype} D{D} bs{bs}")
    assert gpu.get_status(clear=True) == 0


def test_many_short_sequences_per_cta(gpu, one_tile_form):
    """600 sequences of 1 to 40 new tokens (each one item whose tile B is
    empty; 4800 items over the persistent grid, so every CTA claims many of
    them back to back) on prefixes of 0 to 700 tokens."""
    rng = np.random.default_rng(7200)
    B = 600
    prefixes = [int(x) for x in rng.integers(0, 700, B)]
    qlens = [int(x) for x in rng.integers(1, 41, B)]
    c = prefill_case(7200, "bfloat16", 32, 8, 128, "paged", 16, prefixes, qlens)
    assert_close(run(c), ref(c), ATOL_NS, RTOL_NS, "600 short sequences")
    assert gpu.get_status(clear=True) == 0


def test_two_tile_windows_and_long_rows(gpu, one_tile_form):
    """Sliding windows narrower than a pair's row span (tile B's rows start past
    keys tile A needs) and a 2000-token chunk, against the one-tile kernel."""
    c = prefill_case(7300, "bfloat16", 28, 4, 128, "paged", 32, [1000, 0, 64], [2000, 300, 900])
    for window in (None, 100, 700):
        r = ref(c, window=window)
        assert_close(run(c, window=window), r, ATOL_NS, RTOL_NS, f"two-tile window {window}")
        assert_close(one_tile_form(lambda: run(c, window=window)), r, ATOL_NS, RTOL_NS, f"one-tile window {window}")
    assert gpu.get_status(clear=True) == 0
