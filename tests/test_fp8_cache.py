"""GPU tests of the one-byte (FP8) KV cache: the quantising append and the
elementwise codec bit-exact against oracle/kv_oracle.py's restatement of
float8.metal / convert_fp8.metal, and the decode against the float64 decode
of the dequantised caches, over formats, query dtypes, head sizes, block
sizes, group sizes, split-K, ALiBi and the edge rules."""

import math

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close
from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray

pytestmark = pytest.mark.gpu


def fp8_case(seed, qdt, num_seqs, hq, hkv, d, bs, lens, fmt="e4m3", k_scale=1 / 32, v_scale=1 / 24):
    """N(0, 1) inputs; the default scales keep |x / scale| well under E4M3's 240."""
    c = cases.paged_batch(seed, "float32", num_seqs, hq, hkv, d, bs, lens)
    nb = c["k_cache"].shape[0]
    c["k_cache"] = np.zeros((nb, hkv, d // 16, bs, 16), np.uint8)
    c["v_cache"] = np.zeros((nb, hkv, d, bs), np.uint8)
    c.update(qdt=qdt, fmt=fmt, k_scale=k_scale, v_scale=v_scale)
    c["q"] = cases.cast(c["q"], qdt)
    return c


def upload(c, kv_dtype="float32"):
    d = dict(q=DeviceArray.from_numpy(c["q"], dtype=c["qdt"]),
             k=DeviceArray.from_numpy(c["k"], dtype=kv_dtype), v=DeviceArray.from_numpy(c["v"], dtype=kv_dtype),
             kc=DeviceArray.from_numpy(c["k_cache"]), vc=DeviceArray.from_numpy(c["v_cache"]),
             tables=DeviceArray.from_numpy(c["block_tables"]), lens=DeviceArray.from_numpy(c["context_lens"]),
             slots=DeviceArray.from_numpy(c["slot_mapping"]))
    mk.reshape_and_cache_fp8(d["k"], d["v"], d["kc"], d["vc"], d["slots"], c["k_scale"], c["v_scale"], c["fmt"])
    return d


def oracle_caches(c, kv_dtype="float32"):
    kc, vc = c["k_cache"].copy(), c["v_cache"].copy()
    k = kv_oracle.round_to(c["k"], kv_dtype)
    v = kv_oracle.round_to(c["v"], kv_dtype)
    return kv_oracle.reshape_and_cache_fp8(k, v, kc, vc, c["slot_mapping"], c["k_scale"], c["v_scale"], c["fmt"])


def decode(c, d, partition_size=0, alibi=None, max_seq_len=None):
    return mk.paged_attention_fp8(d["q"], d["kc"], d["vc"], d["tables"], d["lens"], c["num_kv_heads"], c["scale"],
                                  c["block_size"], max_seq_len or c["max_seq_len"], alibi, k_scale=c["k_scale"],
                                  v_scale=c["v_scale"], fp8_format=c["fmt"], partition_size=partition_size).to_numpy()


def ref_decode(c, kc, vc, alibi=None, max_seq_len=None):
    return kv_oracle.paged_attention_fp8(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                         c["scale"], c["block_size"], max_seq_len or c["max_seq_len"], c["k_scale"],
                                         c["v_scale"], c["fmt"], alibi)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("kv_dtype", ["float32", "float16", "bfloat16"])
def test_append_is_bit_exact(gpu, fmt, kv_dtype):
    c = fp8_case(6000, "bfloat16", 3, 8, 2, 128, 16, [5, 77, 300], fmt)
    d = upload(c, kv_dtype)
    kc, vc = oracle_caches(c, kv_dtype)
    np.testing.assert_array_equal(d["kc"].to_numpy(), kc)
    np.testing.assert_array_equal(d["vc"].to_numpy(), vc)
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("qdt", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_decode_matrix(gpu, fmt, qdt, D, bs):
    c = fp8_case(6100 + D + bs, qdt, 3, 8, 2, D, bs, [1, 37, 300], fmt)
    d = upload(c)
    kc, vc = oracle_caches(c)
    ref = ref_decode(c, kc, vc)
    assert_close(decode(c, d), ref, ATOL_NS, RTOL_NS, f"{fmt} {qdt} D{D} bs{bs}")
    assert_close(decode(c, d, partition_size=64), ref, ATOL_NS, RTOL_NS, f"{fmt} {qdt} D{D} bs{bs} split")


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (28, 4), (32, 4), (32, 2), (16, 1)])
def test_group_sizes(gpu, Hq, Hkv):
    c = fp8_case(6200 + Hq + Hkv, "bfloat16", 3, Hq, Hkv, 128, 16, [200, 33, 1500])
    d = upload(c)
    kc, vc = oracle_caches(c)
    assert_close(decode(c, d), ref_decode(c, kc, vc), ATOL_NS, RTOL_NS, f"G={Hq // Hkv}")


def test_alibi_zero_rows_and_max_seq_len(gpu):
    lens = [0, 1, 17, 300, 2000, 0]
    c = fp8_case(6300, "float16", len(lens), 8, 2, 128, 16, [max(x, 1) for x in lens])
    c["context_lens"] = np.asarray(lens, np.int32)
    d = upload(c)
    kc, vc = oracle_caches(c)
    slopes = (2.0 ** -np.arange(1, 9)).astype(np.float32)
    al = DeviceArray.from_numpy(slopes)
    for psize in (0, 256):
        out = decode(c, d, psize, alibi=al)
        assert not out[0].any() and not out[5].any()
        assert_close(out, ref_decode(c, kc, vc, alibi=slopes), ATOL_NS, RTOL_NS, f"alibi P={psize}")
    out = decode(c, d, max_seq_len=1024)
    assert not out[4].any()
    assert_close(out, ref_decode(c, kc, vc, max_seq_len=1024), ATOL_NS, RTOL_NS, "max_seq_len")


def test_reference_inf_and_nan_codes(gpu):
    """E4M3's all-ones exponent is Inf/NaN in float8.metal (the hardware's
    E4M3FN reads those codes as 256..448): a V code 0x78 in context gives an
    infinite output, 0x79 a NaN, exactly like the oracle's decode."""
    c = fp8_case(6400, "bfloat16", 1, 4, 1, 64, 16, [16])
    d = upload(c)
    kc, vc = oracle_caches(c)
    blk = c["block_tables"][0, 0]
    vc[blk, 0, 3, 5] = 0x78  # dim 3 of token 5: +Inf
    vc[blk, 0, 9, 2] = 0x79  # dim 9 of token 2: NaN
    d["vc"] = DeviceArray.from_numpy(vc)
    out = decode(c, d)
    ref = ref_decode(c, kc, vc)
    assert np.isposinf(out[0, :, 3]).all() and np.isposinf(ref[0, :, 3]).all()
    assert np.isnan(out[0, :, 9]).all() and np.isnan(ref[0, :, 9]).all()
    keep = [i for i in range(64) if i not in (3, 9)]
    assert_close(out[:, :, keep], ref[:, :, keep], ATOL_NS, RTOL_NS, "finite dims")


def test_nan_garbage_beyond_context_is_never_used(gpu):
    c = fp8_case(6500, "float16", 2, 8, 2, 128, 16, [20, 40])
    c["k_cache"][:] = 0x7F
    c["v_cache"][:] = 0x7F
    d = upload(c)
    assert np.isfinite(decode(c, d)).all()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_convert_fp8_all_directions(gpu, fmt):
    rng = np.random.default_rng(66)
    x = (rng.standard_normal((7, 33)) * 3).astype(np.float32)
    x[0, :4] = [np.inf, -np.inf, np.nan, 1e9]
    scale = 0.25
    codes = DeviceArray.zeros((7, 33), "uint8")
    mk.convert_fp8(codes, DeviceArray.from_numpy(x), scale, fmt)
    ref_codes = kv_oracle.quantize(x, scale, fmt)
    np.testing.assert_array_equal(codes.to_numpy(), ref_codes)
    for dt in ("float32", "float16", "bfloat16"):
        out = DeviceArray.empty((7, 33), dt)
        mk.convert_fp8(out, codes, scale, fmt)
        ref = kv_oracle.round_to(kv_oracle.dequantize(ref_codes, scale, fmt), dt)
        got = out.to_numpy().astype(np.float32) if dt != "bfloat16" else out.to_numpy()
        np.testing.assert_array_equal(np.nan_to_num(got.astype(np.float32), nan=7.0),
                                      np.nan_to_num(ref.astype(np.float32), nan=7.0))
    resc = DeviceArray.zeros((7, 33), "uint8")
    mk.convert_fp8(resc, codes, 2.0, fmt)
    np.testing.assert_array_equal(resc.to_numpy(),
                                  kv_oracle.float_to_fp8(kv_oracle.fp8_to_float(ref_codes, fmt) * np.float32(2.0), fmt))


def test_config2_shape(gpu):
    """Config 2's shape (32 sequences here, U[512, 4096] tokens, 32/8 heads) in
    E4M3: the decode matches the float64 decode of the dequantised caches."""
    rng = np.random.default_rng(2024)
    lens = rng.integers(512, 4097, size=32)
    c = fp8_case(6600, "bfloat16", 32, 32, 8, 128, 16, lens)
    d = upload(c)
    out = decode(c, d)
    kc, vc = oracle_caches(c)
    pick = [0, 31]
    ref = kv_oracle.paged_attention_fp8(c["q"][pick], kc, vc, c["block_tables"][pick], c["context_lens"][pick], 8,
                                        c["scale"], 16, c["max_seq_len"], c["k_scale"], c["v_scale"], "e4m3")
    assert_close(out[pick], ref, ATOL_NS, RTOL_NS, "oracle subset")
