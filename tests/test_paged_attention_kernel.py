"""GPU parity tests of the paged-KV kernels through the C ABI.

Mirrors the reference's tests/test_paged_attention_kernel.py one for one
(shapes, edge cases, messages), adds the golden fixtures made from the
reference's own NumPy oracles, and extends coverage to the full dtype /
head-size / block-size / group-size matrix, split-K, ALiBi and the bounds
checks.  Oracle: oracle/kv_oracle.py (float64)."""

import math
import os

import numpy as np
import pytest

import cases
from helpers import (ATOL_NS, RTOL_NS, assert_close, fill_cache, oracle_fill, tolerance, upload_case)
from oracle import c_oracle, kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray

pytestmark = pytest.mark.gpu


def run_v1(d, c, max_seq_len=None, alibi=None):
    return mk.paged_attention_v1(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                 c["num_kv_heads"], c["scale"], c["block_size"],
                                 max_seq_len or c["max_seq_len"], alibi)


def run_v2(d, c, partition_size=512, max_seq_len=None, alibi=None):
    return mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                 c["num_kv_heads"], c["scale"], c["block_size"],
                                 max_seq_len or c["max_seq_len"], alibi, partition_size=partition_size)


# ---- the reference's own tests ------------------------------------------------

def test_reshape_and_cache(gpu, golden):
    """test_paged_attention_kernel.py:190-210 (f32 K/V into an fp16 cache), bit-exact."""
    c = cases.ref_setup_data()
    d = upload_case(c)
    kc, vc = fill_cache(d)
    np.testing.assert_array_equal(kc.to_numpy(), golden["ref_setup/k_cache"])
    np.testing.assert_array_equal(vc.to_numpy(), golden["ref_setup/v_cache"])
    assert gpu.get_status(clear=True) == 0


def test_paged_attention_v1(gpu, golden):
    """test_paged_attention_kernel.py:212-246 (atol 5e-3 there; tighter here)."""
    c = cases.ref_setup_data()
    d = upload_case(c)
    fill_cache(d)
    out = run_v1(d, c, max_seq_len=64).to_numpy()
    np.testing.assert_allclose(out, golden["ref_setup/attn"], atol=5e-3)
    assert_close(out, golden["ref_setup/attn"], 1e-4, 1e-4, "ref_setup")


@pytest.mark.parametrize("head_dim", [32, 128])
@pytest.mark.parametrize("block_size", [8, 16])
def test_various_shapes(gpu, golden, head_dim, block_size):
    """test_paged_attention_kernel.py:248-282."""
    c = cases.ref_various(head_dim, block_size)
    d = upload_case(c)
    fill_cache(d)
    out = run_v1(d, c, max_seq_len=16).to_numpy()
    ref = golden[f"ref_various_{head_dim}_{block_size}/attn"]
    np.testing.assert_allclose(out, ref, atol=5e-3)
    assert_close(out, ref, 1e-4, 1e-4, "various")


def test_context_longer_than_legacy_2048_limit(gpu, golden):
    """test_paged_attention_kernel.py:284-330 (uint32 tables and lengths)."""
    c = cases.ref_legacy_2048()
    d = upload_case(c)
    assert d["block_tables"].dtype == "uint32" and d["context_lens"].dtype == "uint32"
    fill_cache(d)
    np.testing.assert_array_equal(d["k_cache"].to_numpy(), golden["ref_legacy_2048/k_cache"])
    out = run_v1(d, c, max_seq_len=2112).to_numpy()
    np.testing.assert_allclose(out, golden["ref_legacy_2048/attn"], atol=5e-3)
    assert_close(out, golden["ref_legacy_2048/attn"], 1e-4, 1e-4, "legacy 2048")


def _tiny(context_len, max_seq_len):
    rng = np.random.default_rng(5)
    q = DeviceArray.from_numpy(rng.standard_normal((1, 2, 32), dtype=np.float32))
    kc = DeviceArray.zeros((1, 1, 4, 16, 8), "float16")
    vc = DeviceArray.zeros((1, 1, 32, 16), "float16")
    bt = DeviceArray.from_numpy(np.array([[0]], np.int32))
    cl = DeviceArray.from_numpy(np.array([context_len], np.int32))
    return mk.paged_attention_v1(q, kc, vc, bt, cl, 1, 1.0 / math.sqrt(32), 16, max_seq_len)


def test_empty_context_returns_zero(gpu):
    """test_paged_attention_kernel.py:332-354: exact zeros."""
    out = _tiny(0, 16).to_numpy()
    np.testing.assert_array_equal(out, np.zeros(out.shape))


def test_context_over_max_seq_len_returns_zero(gpu):
    """test_paged_attention_kernel.py:356-378."""
    out = _tiny(16, 8).to_numpy()
    np.testing.assert_array_equal(out, np.zeros(out.shape))


def test_rejects_max_seq_len_beyond_block_table_capacity(gpu):
    """test_paged_attention_kernel.py:380-398."""
    q = DeviceArray.zeros((1, 2, 32), "float32")
    kc = DeviceArray.zeros((2, 1, 4, 16, 8), "float16")
    vc = DeviceArray.zeros((2, 1, 32, 16), "float16")
    with pytest.raises(ValueError, match="block table capacity"):
        mk.paged_attention_v1(q, kc, vc, np.array([[0]], np.int32), np.array([1], np.int32), 1, 1.0, 16, 17)


# ---- golden: BASELINE.json config 1 -----------------------------------------------

@pytest.mark.parametrize("name,seed,dtype", [("config1_fp16", 11, "float16"), ("config1_bf16", 12, "bfloat16")])
def test_config1_against_reference_oracle(gpu, golden, name, seed, dtype):
    c = cases.config1(seed=seed, dtype=dtype)
    d = upload_case(c)
    kc, vc = fill_cache(d)
    # cache contents bit-exact with the reference oracle's reshape_and_cache
    kraw = kc.to_numpy(raw=True) if dtype == "bfloat16" else kc.to_numpy()
    vraw = vc.to_numpy(raw=True) if dtype == "bfloat16" else vc.to_numpy()
    if dtype == "bfloat16":
        kraw = kv_oracle.bf16_bits_to_f32(kraw).reshape(kraw.shape)
        vraw = kv_oracle.bf16_bits_to_f32(vraw).reshape(vraw.shape)
    assert cases.digest(kraw) == str(golden[f"{name}/k_cache_sha"])
    assert cases.digest(vraw) == str(golden[f"{name}/v_cache_sha"])
    ref = golden[f"{name}/attn"].astype(np.float64)
    for fn in (run_v1, run_v2):
        out = fn(d, c).to_numpy()
        np.testing.assert_allclose(out, ref, atol=5e-3)
        assert_close(out, ref, ATOL_NS, RTOL_NS, f"{name} {fn.__name__}")
    assert gpu.get_status(clear=True) == 0


# ---- coverage beyond the reference tests ---------------------------------------------

PAIRS = [("float32", "float32"), ("bfloat16", "bfloat16"), ("float16", "float16"), ("float32", "float16"),
         ("float32", "bfloat16")]


@pytest.mark.parametrize("qd,cd", PAIRS)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_dtype_headsize_blocksize_matrix(gpu, qd, cd, D, bs):
    c = cases.paged_batch(100 + D + bs, "float32", 3, 8, 2, D, bs, [1, 37, 300], cache_dtype=cd)
    d = upload_case(c, cache_dtype=cd, q_dtype=qd)
    fill_cache(d)
    kc, vc = oracle_fill(c, cd)
    qv = kv_oracle.round_to(c["q"], qd)
    ref = kv_oracle.paged_attention_v1(qv, kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], bs,
                                       c["max_seq_len"])
    atol, rtol = tolerance(qd)
    for fn in (run_v1, lambda d_, c_: run_v2(d_, c_, partition_size=64)):
        assert_close(fn(d, c).to_numpy(), ref, atol, rtol, f"{qd}/{cd} D{D} bs{bs}")


@pytest.mark.parametrize("D", [32, 80, 96, 112, 120, 192, 256])
def test_other_head_sizes(gpu, D):
    c = cases.paged_batch(7 + D, "bfloat16", 2, 4, 2, D, 16, [45, 130])
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16,
                                       c["max_seq_len"])
    assert_close(run_v1(d, c).to_numpy(), ref, ATOL_NS, RTOL_NS, f"D{D}")


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (16, 4), (28, 4), (32, 4), (32, 2), (64, 2), (32, 1)])
def test_group_sizes(gpu, Hq, Hkv):
    c = cases.paged_batch(Hq * 10 + Hkv, "bfloat16", 2, Hq, Hkv, 128, 16, [200, 33])
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], Hkv, c["scale"], 16,
                                       c["max_seq_len"])
    for fn in (run_v1, lambda d_, c_: run_v2(d_, c_, partition_size=64)):
        assert_close(fn(d, c).to_numpy(), ref, ATOL_NS, RTOL_NS, f"G={Hq // Hkv}")


def test_alibi(gpu):
    c = cases.paged_batch(31, "float16", 3, 8, 2, 128, 16, [17, 200, 64])
    d = upload_case(c)
    fill_cache(d)
    slopes = (2.0 ** -np.arange(1, 9)).astype(np.float32)
    kc, vc = oracle_fill(c, "float16")
    ref = kv_oracle.paged_attention_v1(c["q"].astype(np.float32), kc, vc, c["block_tables"], c["context_lens"], 2,
                                       c["scale"], 16, c["max_seq_len"], slopes)
    al = DeviceArray.from_numpy(slopes)
    assert_close(run_v1(d, c, alibi=al).to_numpy(), ref, ATOL_NS, RTOL_NS, "alibi v1")
    assert_close(run_v2(d, c, partition_size=32, alibi=al).to_numpy(), ref, ATOL_NS, RTOL_NS, "alibi v2")


def test_splitk_long_context_against_c_oracle(gpu):
    """A reduced config 3: batch 1, 64 q / 8 kv heads, block 32, 16k tokens in
    permuted blocks, 512-token partitions + LSE reduce."""
    c = cases.paged_batch(303, "bfloat16", 1, 64, 8, 128, 32, [16384 - 5])
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    bits = kv_oracle.f32_to_bf16_bits
    ref = c_oracle.paged_attention(bits(c["q"]), "bfloat16", bits(kc), bits(vc), "bfloat16", c["block_tables"],
                                   c["context_lens"], 8, c["scale"], c["max_seq_len"])
    out2 = run_v2(d, c).to_numpy()
    out1 = run_v1(d, c).to_numpy()
    assert_close(out2, ref, ATOL_NS, RTOL_NS, "split-K")
    assert_close(out1, ref, ATOL_NS, RTOL_NS, "single pass")


def test_mixed_lengths_and_zero_rows_in_one_batch(gpu):
    lens = [0, 1, 15, 16, 17, 511, 512, 513, 1000]
    c = cases.paged_batch(77, "bfloat16", len(lens), 16, 4, 128, 16, [max(x, 1) for x in lens])
    c["context_lens"] = np.array(lens, np.int32)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 4, c["scale"], 16,
                                       c["max_seq_len"])
    for fn in (run_v1, lambda d_, c_: run_v2(d_, c_, partition_size=256)):
        out = fn(d, c).to_numpy()
        assert not out[0].any()
        assert_close(out, ref, ATOL_NS, RTOL_NS, "mixed")


def test_short_bf16_sequences_meet_the_tolerance(gpu):
    """64 sequences of 1..64 tokens: with few tokens and nearly cancelling V
    rows the output is sensitive to how P is rounded for the P.V product."""
    c = cases.paged_batch(2501, "bfloat16", 64, 32, 2, 128, 16, list(range(1, 65)))
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16,
                                       c["max_seq_len"])
    for fn in (run_v1, lambda d_, c_: run_v2(d_, c_, partition_size=32)):
        assert_close(fn(d, c).to_numpy(), ref, ATOL_NS, RTOL_NS, "short bf16")


def test_nan_garbage_beyond_context_is_never_used(gpu):
    """Tokens past context_len in the last block hold NaN: they must not leak."""
    c = cases.paged_batch(88, "float16", 2, 8, 2, 128, 16, [20, 40])
    c["k_cache"][:] = np.nan
    c["v_cache"][:] = np.nan
    d = upload_case(c)
    fill_cache(d)
    out = run_v1(d, c).to_numpy()
    assert np.isfinite(out).all()
    out2 = run_v2(d, c, partition_size=32).to_numpy()
    assert np.isfinite(out2).all()


# ---- append / gather coverage --------------------------------------------------------

@pytest.mark.parametrize("kvd,cd", PAIRS)
@pytest.mark.parametrize("slot_dtype", [np.int32, np.int64])
def test_reshape_and_cache_matrix_bit_exact(gpu, kvd, cd, slot_dtype):
    rng = np.random.default_rng(3)
    T, H, D, bs, nb = 70, 4, 64, 16, 12
    k = rng.standard_normal((T, H, D), dtype=np.float32)
    v = rng.standard_normal((T, H, D), dtype=np.float32)
    slots = rng.permutation(nb * bs)[:T].astype(slot_dtype)
    slots[::9] = -1
    x = 16 // (4 if cd == "float32" else 2)
    kc = DeviceArray.zeros((nb, H, D // x, bs, x), cd)
    vc = DeviceArray.zeros((nb, H, D, bs), cd)
    mk.reshape_and_cache(DeviceArray.from_numpy(k, dtype=kvd), DeviceArray.from_numpy(v, dtype=kvd), kc, vc,
                         DeviceArray.from_numpy(slots))
    kin = kv_oracle.round_to(kv_oracle.round_to(k, kvd), cd)
    vin = kv_oracle.round_to(kv_oracle.round_to(v, kvd), cd)
    rk = np.zeros((nb, H, D // x, bs, x), np.float32)
    rv = np.zeros((nb, H, D, bs), np.float32)
    kv_oracle.reshape_and_cache(kin, vin, rk, rv, slots)
    np.testing.assert_array_equal(kc.to_numpy().astype(np.float32), rk)
    np.testing.assert_array_equal(vc.to_numpy().astype(np.float32), rv)


def test_reshape_and_cache_flash_and_strided_source(gpu):
    rng = np.random.default_rng(4)
    T, H, D, bs, nb = 50, 4, 128, 16, 8
    src = rng.standard_normal((H, T, D), dtype=np.float32)  # head-major source, read through strides
    k = DeviceArray.from_numpy(src, dtype="bfloat16").transpose(1, 0, 2)
    v = DeviceArray.from_numpy(src * 2, dtype="bfloat16").transpose(1, 0, 2)
    slots = rng.permutation(nb * bs)[:T].astype(np.int32)
    kc = DeviceArray.zeros((nb, bs, H, D), "bfloat16")
    vc = DeviceArray.zeros((nb, bs, H, D), "bfloat16")
    mk.reshape_and_cache_flash(k, v, kc, vc, slots)
    rk = np.zeros((nb, bs, H, D), np.float32)
    rv = np.zeros((nb, bs, H, D), np.float32)
    kv_oracle.reshape_and_cache_flash(kv_oracle.round_to(src.transpose(1, 0, 2), "bfloat16"),
                                      kv_oracle.round_to(src.transpose(1, 0, 2) * 2, "bfloat16"), rk, rv, slots)
    np.testing.assert_array_equal(kc.to_numpy(), rk)
    np.testing.assert_array_equal(vc.to_numpy(), rv)


def test_gather_kv_bit_exact(gpu):
    rng = np.random.default_rng(6)
    S, H, D = 300, 8, 128
    kb = rng.standard_normal((S, H, D), dtype=np.float32).astype(np.float16)
    vb = rng.standard_normal((S, H, D), dtype=np.float32).astype(np.float16)
    idx = rng.integers(0, S, size=257).astype(np.int64)
    k, v = mk.gather_kv(DeviceArray.from_numpy(kb), DeviceArray.from_numpy(vb), DeviceArray.from_numpy(idx))
    rk, rv = kv_oracle.pool_fetch(kb, vb, idx)
    np.testing.assert_array_equal(k.to_numpy(), rk)
    np.testing.assert_array_equal(v.to_numpy(), rv)


# ---- bounds checks (no fault: skipped and flagged) -----------------------------------

def test_out_of_range_slot_is_skipped_and_flagged(gpu):
    gpu.get_status(clear=True)
    kc = DeviceArray.zeros((2, 1, 4, 16, 8), "float16")
    vc = DeviceArray.zeros((2, 1, 32, 16), "float16")
    k = DeviceArray.from_numpy(np.ones((3, 1, 32), np.float16))
    mk.reshape_and_cache(k, k, kc, vc, np.array([1, 32, 5], np.int32))  # slot 32 = block 2 of 2
    assert gpu.get_status(clear=True) & _lib.STATUS_SLOT_OOB
    got = vc.to_numpy()
    assert got[0, 0, :, 1].all() and got[0, 0, :, 5].all() and got.sum() == 2 * 32


def test_out_of_range_block_is_skipped_and_flagged(gpu):
    gpu.get_status(clear=True)
    c = cases.paged_batch(9, "float16", 1, 4, 2, 64, 16, [40])
    d = upload_case(c)
    fill_cache(d)
    bad = c["block_tables"].copy()
    bad[0, 1] = 10_000
    out = mk.paged_attention_v1(d["q"], d["k_cache"], d["v_cache"], DeviceArray.from_numpy(bad),
                                d["context_lens"], 2, c["scale"], 16, c["max_seq_len"])
    assert np.isfinite(out.to_numpy()).all()
    assert gpu.get_status(clear=True) & _lib.STATUS_BLOCK_OOB


def test_torch_tensors_via_dlpack(gpu):
    torch = pytest.importorskip("torch")
    c = cases.config1(dtype="float16")
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(dev) for k in
         ("q", "k", "v", "k_cache", "v_cache", "block_tables", "context_lens", "slot_mapping")}
    mk.reshape_and_cache(t["k"], t["v"], t["k_cache"], t["v_cache"], t["slot_mapping"])
    out = mk.paged_attention_v1(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"], 8,
                                c["scale"], 16, c["max_seq_len"])
    torch.cuda.synchronize()
    golden = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    assert_close(out.to_numpy(), golden["config1_fp16/attn"].astype(np.float64), ATOL_NS, RTOL_NS, "torch")
    back = torch.from_dlpack(out)
    assert back.shape == (8, 32, 128) and back.dtype == torch.float16


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_tensor_core_and_generic_kernels_agree(gpu, monkeypatch, dtype, bs):
    """The same inputs through both decode kernels (KVC_DECODE_KERNEL=generic
    forces the CUDA-core one) agree with each other and with the oracle."""
    c = cases.paged_batch(500 + bs, dtype, 5, 28, 4, 128, bs, [3, 64, 65, 700, 2049])
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(kv_oracle.round_to(c["q"], dtype), kc, vc, c["block_tables"],
                                       c["context_lens"], 4, c["scale"], bs, c["max_seq_len"])
    fast = run_v1(d, c).to_numpy()
    fast2 = run_v2(d, c, partition_size=128).to_numpy()
    monkeypatch.setenv("KVC_DECODE_KERNEL", "generic")
    slow = run_v1(d, c).to_numpy()
    slow2 = run_v2(d, c, partition_size=128).to_numpy()
    monkeypatch.delenv("KVC_DECODE_KERNEL")
    for name, out in (("mma v1", fast), ("mma v2", fast2), ("generic v1", slow), ("generic v2", slow2)):
        assert_close(out, ref, ATOL_NS, RTOL_NS, name)
    assert_close(fast, slow, ATOL_NS, RTOL_NS, "mma vs generic")


@pytest.mark.parametrize("variant", ["2x3", "2x2", "4x3x16", "4x3x16t", "2x2x32t", "4x3x16s", "2x2x32s", "3x2x32s", "2x3x32s"])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_ring_variants(gpu, monkeypatch, variant, bs):
    """Every (warps x stages) ring configuration of the tensor-core kernel."""
    monkeypatch.setenv("KVC_MMA_CONFIG", variant)
    c = cases.paged_batch(900 + bs, "bfloat16", 6, 32, 8, 128, bs, [1, 31, 33, 128, 517, 1999])
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 8, c["scale"], bs,
                                       c["max_seq_len"])
    assert_close(run_v1(d, c).to_numpy(), ref, ATOL_NS, RTOL_NS, f"{variant} v1")
    assert_close(run_v2(d, c, partition_size=256).to_numpy(), ref, ATOL_NS, RTOL_NS, f"{variant} v2")


def test_decode_step_replays_as_cuda_graph(gpu):
    """append + single-pass + split-K decode captured once, replayed twice: same results as eager."""
    from sglang_mlx_b200.device_array import Graph, Stream

    c = cases.paged_batch(1234, "bfloat16", 4, 32, 8, 128, 16, [100, 700, 33, 1500])
    d = upload_case(c)
    fill_cache(d)
    st = Stream()
    o1 = DeviceArray.empty(d["q"].shape, "bfloat16")
    o2 = DeviceArray.empty(d["q"].shape, "bfloat16")
    ws = mk.splitk_workspace(4, 32, 128, c["max_seq_len"], 256)
    k_new = DeviceArray.from_numpy(np.ones((4, 8, 128), np.float32), dtype="bfloat16")
    slots = DeviceArray.from_numpy(np.array([c["block_tables"][i, 0] * 16 for i in range(4)], np.int32))

    def work():
        mk.reshape_and_cache(k_new, k_new, d["k_cache"], d["v_cache"], slots, stream=st)
        mk.paged_attention_v1(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 8,
                              c["scale"], 16, c["max_seq_len"], out=o1, stream=st)
        mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 8,
                              c["scale"], 16, c["max_seq_len"], partition_size=256, workspace=ws, out=o2, stream=st)

    work()  # eager first (sets kernel attributes)
    st.synchronize()
    e1, e2 = o1.to_numpy(), o2.to_numpy()
    g = Graph.capture(st, work)
    for _ in range(2):
        o1.fill_zero(stream=st)
        o2.fill_zero(stream=st)
        g.replay(st)
        st.synchronize()
        np.testing.assert_array_equal(o1.to_numpy(), e1)
        np.testing.assert_array_equal(o2.to_numpy(), e2)
    assert_close(e2, e1, ATOL_NS, RTOL_NS, "split vs single pass")
