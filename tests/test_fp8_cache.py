"""GPU tests of the one-byte (FP8) KV cache: the codec bit-exact against the
reference's own float8.metal functions (vectors and an exhaustive 2^32 sweep
digest from tests/golden/make_fp8_golden.py), the quantising append and the
elementwise codec bit-exact against oracle/kv_oracle.py's restatement of
float8.metal / convert_fp8.metal, and the decode against the float64 decode
of the dequantised caches, over formats, query dtypes, head sizes, block
sizes, group sizes, split-K, ALiBi and the edge rules."""

import hashlib
import math
import os

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


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e4m3-sat", "e5m2-sat"])
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


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fp8_ref.npz")


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_codec_matches_reference_vectors(gpu, fmt):
    """The device codec against the reference's float8.metal functions run on
    the host: encode of every bfloat16 pattern, every float16 value and 2^17
    seeded float32 patterns (kvc_convert_fp8 with scale 1), decode of all 256
    codes; the "-sat" format against the oracle's restatement of it."""
    import make_fp8_golden as g

    ref = np.load(GOLDEN)
    x = g.enc_inputs()
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(ref["enc_inputs_sha256"])
    f = x.view(np.float32)
    src = DeviceArray.from_numpy(f)
    for name, want in ((fmt, ref[f"enc_{fmt}"]), (fmt + "-sat", kv_oracle.float_to_fp8(f, fmt + "-sat"))):
        codes = DeviceArray.zeros(f.shape, "uint8")
        mk.convert_fp8(codes, src, 1.0, name)
        got = codes.to_numpy()
        nan_in = np.isnan(f)
        # NaN inputs: a NaN code either way (the division by the scale may drop a NaN's sign)
        top = 0x78 if fmt == "e4m3" else 0x7C
        assert ((got[nan_in] & top) == top).all() and ((got[nan_in] & ~np.uint8(0x80 | top)) != 0).all()
        np.testing.assert_array_equal(got[~nan_in], want[~nan_in], err_msg=name)
    dec = DeviceArray.empty((256,), "float32")
    mk.convert_fp8(dec, DeviceArray.from_numpy(np.arange(256, dtype=np.uint8)), 1.0, fmt)
    got = dec.to_numpy()
    want = ref[f"dec_{fmt}"].view(np.float32)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    np.testing.assert_array_equal(got[~np.isnan(got)], want[~np.isnan(want)])
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_encoder_exhaustive_sweep(gpu, fmt):
    """The device encoder on every float32 bit pattern 0 .. 2^32 - 1, hashed in
    order: equal to the SHA-256 of the reference encoder's codes (+-Inf where
    that code's shift is undefined).  NaN inputs are checked to give NaN codes
    and then hashed as the reference codes them (sign | all-ones | 1)."""
    torch = pytest.importorskip("torch")
    ref = np.load(GOLDEN)
    dev = torch.device("cuda", 0)
    top = 0x78 if fmt == "e4m3" else 0x7C
    n = 1 << 26
    h = hashlib.sha256()
    codes = DeviceArray.zeros((n,), "uint8")
    codes_t = torch.from_dlpack(codes)
    starts = list(range(0, 1 << 31, n)) + list(range(-(1 << 31), 0, n))  # bit patterns 0 .. 2^32 - 1 in order
    for start in starts:
        bits = torch.arange(start, start + n, dtype=torch.int32, device=dev)
        x = bits.view(torch.float32)
        mk.convert_fp8(codes, x, 1.0, fmt)
        c = codes_t.to(torch.int32)
        nan_in = torch.isnan(x)
        bad = nan_in & (((c & top) != top) | ((c & ~(0x80 | top)) == 0))
        assert not bool(bad.any()), f"non-NaN code for a NaN input near pattern {start & 0xFFFFFFFF:#x}"
        want_nan = ((bits >> 31) & 1) * 0x80 | top | 1
        c = torch.where(nan_in, want_nan, c)
        h.update(c.to(torch.uint8).cpu().numpy().tobytes())
    torch.cuda.synchronize()
    assert h.hexdigest() == str(ref[f"sweep_sha256_{fmt}"])
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_planned_fp8_decode(gpu, fmt):
    """The planned split-K over one-byte caches (kvc_paged_attention_fp8_planned)
    equals the float64 decode of the dequantised caches, with zero-length and
    over-long sequences in the batch."""
    lens = [0, 1, 100, 700, 2500, 3100, 40]
    c = fp8_case(6700, "bfloat16", len(lens), 8, 2, 128, 16, lens, fmt)
    d = upload(c)
    kc, vc = oracle_caches(c)
    for P, msl in ((512, None), (1024, 3072)):
        plan = mk.make_decode_plan(d["lens"], 2, msl or c["max_seq_len"], P)
        out = mk.paged_attention_fp8(d["q"], d["kc"], d["vc"], d["tables"], d["lens"], 2, c["scale"], 16,
                                     msl or c["max_seq_len"], k_scale=c["k_scale"], v_scale=c["v_scale"],
                                     fp8_format=fmt, plan=plan).to_numpy()
        assert_close(out, ref_decode(c, kc, vc, max_seq_len=msl), ATOL_NS, RTOL_NS, f"planned fp8 P={P}")
        assert not out[0].any()
    assert gpu.get_status(clear=True) == 0
