"""CPU oracle pinned against the reference's own outputs (tests/golden/golden.npz,
made by tests/golden/make_golden.py from the reference's NumPy oracles and its
MHATokenPool).  No GPU."""

import hashlib
import os

import numpy as np
import pytest

import cases
from oracle import c_oracle, kv_oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REF_CASES = {
    "ref_setup": cases.ref_setup_data,
    "ref_various_32_8": lambda: cases.ref_various(32, 8),
    "ref_various_32_16": lambda: cases.ref_various(32, 16),
    "ref_various_128_8": lambda: cases.ref_various(128, 8),
    "ref_various_128_16": lambda: cases.ref_various(128, 16),
    "ref_legacy_2048": cases.ref_legacy_2048,
    "config1_fp16": lambda: cases.config1(dtype="float16"),
    "config1_bf16": lambda: cases.config1(seed=12, dtype="bfloat16"),
}


def _fill(c):
    kc, vc = c["k_cache"].copy(), c["v_cache"].copy()
    T = c["k"].shape[0]
    k = c["k"].astype(kc.dtype)
    v = c["v"].astype(vc.dtype)
    return kv_oracle.reshape_and_cache(k, v, kc, vc, c["slot_mapping"][:T])


@pytest.mark.parametrize("name", list(REF_CASES))
def test_inputs_match_fixture(name, golden):
    c = REF_CASES[name]()
    assert cases.digest(c["q"], c["k"], c["v"], c["block_tables"], c["context_lens"], c["slot_mapping"]) == str(
        golden[f"{name}/inputs_sha"]), "seeded inputs drifted from the fixture"


@pytest.mark.parametrize("name", list(REF_CASES))
def test_reshape_and_cache_bit_exact(name, golden):
    c = REF_CASES[name]()
    kc, vc = _fill(c)
    assert cases.digest(kc) == str(golden[f"{name}/k_cache_sha"])
    assert cases.digest(vc) == str(golden[f"{name}/v_cache_sha"])
    if f"{name}/k_cache" in golden:
        np.testing.assert_array_equal(kc, golden[f"{name}/k_cache"])
        np.testing.assert_array_equal(vc, golden[f"{name}/v_cache"])


@pytest.mark.parametrize("name", list(REF_CASES))
def test_paged_attention_matches_reference_oracle(name, golden):
    c = REF_CASES[name]()
    kc, vc = _fill(c)
    out = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                       c["scale"], c["block_size"], c["max_seq_len"])
    ref = golden[f"{name}/attn"]
    # The reference oracle rounds its float64 result to the query dtype and has
    # no +1e-6 in the denominator: agree to the output dtype's rounding.
    got = out.astype(ref.dtype)
    tol = 1e-3 if ref.dtype == np.float16 else 1e-5
    np.testing.assert_allclose(got.astype(np.float64), ref.astype(np.float64), rtol=tol, atol=tol)


def test_c_oracle_matches_numpy_oracle():
    c = cases.config1(dtype="float16")
    kc, vc = _fill(c)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                       c["scale"], c["block_size"], c["max_seq_len"])
    got = c_oracle.paged_attention(c["q"], "float16", kc, vc, "float16", c["block_tables"], c["context_lens"],
                                   c["num_kv_heads"], c["scale"], c["max_seq_len"])
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def test_c_oracle_bf16_bits_and_alibi():
    c = cases.config1(seed=12, dtype="bfloat16")
    kc, vc = _fill(c)
    slopes = np.linspace(-0.05, 0.05, c["q"].shape[1]).astype(np.float32)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                       c["scale"], c["block_size"], c["max_seq_len"], slopes)
    bits = lambda a: kv_oracle.f32_to_bf16_bits(a)  # noqa: E731
    got = c_oracle.paged_attention(bits(c["q"]), "bfloat16", bits(kc), bits(vc), "bfloat16", c["block_tables"],
                                   c["context_lens"], c["num_kv_heads"], c["scale"], c["max_seq_len"], slopes)
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def test_c_oracle_reshape_matches_numpy_oracle():
    c = cases.config1(dtype="float16")
    kc1, vc1 = _fill(c)
    kc2, vc2 = c["k_cache"].copy(), c["v_cache"].copy()
    c_oracle.reshape_and_cache(c["k"].astype(np.float16), c["v"].astype(np.float16), kc2, vc2, c["slot_mapping"])
    np.testing.assert_array_equal(kc1, kc2)
    np.testing.assert_array_equal(vc1, vc2)


@pytest.mark.parametrize("psize", [16, 64, 512])
def test_splitk_restatement_equals_single_pass(psize):
    c = cases.config1(dtype="float16")
    kc, vc = _fill(c)
    one = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                       c["scale"], c["block_size"], c["max_seq_len"])
    split, _, _ = kv_oracle.paged_attention_splitk(c["q"], kc, vc, c["block_tables"], c["context_lens"],
                                                   c["num_kv_heads"], c["scale"], c["block_size"], c["max_seq_len"],
                                                   psize)
    np.testing.assert_allclose(split, one, rtol=1e-9, atol=1e-12)


def test_zero_output_rules():
    c = cases.ref_various(32, 16)
    kc, vc = _fill(c)
    for lens, msl in (([0], 16), ([16], 8)):
        out = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], np.array(lens), 2, c["scale"], 16, msl)
        assert not out.any()


def test_pool_store_fetch_matches_reference_pool(golden):
    k_buf = [np.zeros((41, 4, 8), np.float32) for _ in range(2)]
    v_buf = [np.zeros((41, 4, 8), np.float32) for _ in range(2)]
    i = 0
    while f"pool/write{i}/layer" in golden:
        layer = int(golden[f"pool/write{i}/layer"])
        kv_oracle.pool_store(k_buf[layer], v_buf[layer], golden[f"pool/write{i}/idx"], golden[f"pool/write{i}/k"],
                             golden[f"pool/write{i}/v"])
        i += 1
    for layer in (0, 1):
        k, v = kv_oracle.pool_fetch(k_buf[layer], v_buf[layer], golden["pool/fetch_idx"])
        np.testing.assert_array_equal(k, golden[f"pool/fetch{layer}/k"])
        np.testing.assert_array_equal(v, golden[f"pool/fetch{layer}/v"])


def test_bf16_rounding_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.0078125, 1.01171875, -3.0e38, 3.4e38, 1e-40], np.float32)
    bits = kv_oracle.f32_to_bf16_bits(vals)
    back = kv_oracle.bf16_bits_to_f32(bits)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: rounds to even (1.0)
    assert back[1] == 1.0 and back[3] == np.float32(1.015625)
    assert np.isinf(back[5])


def test_copy_blocks_oracle_matches_reference_test():
    """test_paged_attention_kernel.py:400-425 restated on the oracle."""
    keys = [np.arange(24, dtype=np.float32).reshape(4, 2, 3) + layer * 100 for layer in range(2)]
    vals = [k + 1000 for k in keys]
    before_k = [k.copy() for k in keys]
    before_v = [v.copy() for v in vals]
    kv_oracle.copy_blocks(keys, vals, [[0, 2], [1, 3]])
    for layer in range(2):
        ek, ev = before_k[layer].copy(), before_v[layer].copy()
        ek[2], ek[3] = before_k[layer][0], before_k[layer][1]
        ev[2], ev[3] = before_v[layer][0], before_v[layer][1]
        np.testing.assert_array_equal(keys[layer], ek)
        np.testing.assert_array_equal(vals[layer], ev)


def test_swap_blocks_oracle_matches_reference_test():
    """test_paged_attention_kernel.py:427-438 restated on the oracle."""
    src = np.arange(24, dtype=np.float32).reshape(4, 2, 3)
    dst = np.full((4, 2, 3), -1, dtype=np.float32)
    expected = dst.copy()
    expected[2] = src[0]
    expected[1] = src[3]
    np.testing.assert_array_equal(kv_oracle.swap_blocks(src, dst, [[0, 2], [3, 1]]), expected)


@pytest.mark.parametrize("bs", [1, 16])
def test_flash_oracle_equals_paged_oracle(bs):
    """The token-major restatement (paged_attention_flash) on caches filled with
    the same tokens as the vLLM-layout caches gives the same float64 result as
    the golden-pinned paged_attention_v1 restatement."""
    c = cases.paged_batch(77, "float16", 3, 8, 2, 64, 16, [5, 40, 130])
    kc, vc = kv_oracle.reshape_and_cache(c["k"].astype(np.float32), c["v"].astype(np.float32),
                                         c["k_cache"].astype(np.float32), c["v_cache"].astype(np.float32),
                                         c["slot_mapping"])
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16,
                                       c["max_seq_len"])
    nb = c["k_cache"].shape[0]
    if bs == 1:
        fk = np.zeros((nb * 16, 2, 64), np.float32)
        fv = np.zeros_like(fk)
        kv_oracle.reshape_and_cache_flash(c["k"], c["v"], fk, fv, c["slot_mapping"])
        t = np.arange(c["block_tables"].shape[1] * 16)
        tables = c["block_tables"][:, t // 16].astype(np.int64) * 16 + t % 16
    else:
        fk = np.zeros((nb, 16, 2, 64), np.float32)
        fv = np.zeros_like(fk)
        kv_oracle.reshape_and_cache_flash(c["k"], c["v"], fk, fv, c["slot_mapping"])
        tables = c["block_tables"]
    got = kv_oracle.paged_attention_flash(c["q"], fk, fv, tables, c["context_lens"], 2, c["scale"], c["max_seq_len"])
    np.testing.assert_array_equal(got, ref)


def test_fp8_codec_restatement():
    """float8.metal's codecs restated in kv_oracle: checked against torch's OCP
    formats where the formats coincide (every E5M2 code; E4M3 codes below the
    all-ones exponent, which the reference keeps for Inf/NaN) and on known
    answers of the reference's IEEE-style E4M3 (max finite 240) and of its
    encoder's code path (values past 240 through the subnormal branch, a
    subnormal's carry dropped), beside the "-sat" formats' stated behaviour."""
    import torch

    codes = np.arange(256, dtype=np.uint8)
    t5 = torch.from_numpy(codes.copy()).view(torch.float8_e5m2).float().numpy()
    d5 = kv_oracle.fp8_to_float(codes, "e5m2")
    assert np.array_equal(np.isnan(t5), np.isnan(d5)) and np.array_equal(t5[~np.isnan(t5)], d5[~np.isnan(d5)])
    t4 = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    d4 = kv_oracle.fp8_to_float(codes, "e4m3")
    low = ((codes >> 3) & 0xF) != 15
    assert np.array_equal(t4[low], d4[low])
    assert np.isposinf(d4[0x78]) and np.isneginf(d4[0xF8]) and np.isnan(d4[0x79])
    for fmt, dec in (("e4m3", d4), ("e5m2", d5)):  # every finite code survives encode(decode(c))
        fin = np.isfinite(dec)
        for f in (fmt, fmt + "-sat"):
            assert np.array_equal(kv_oracle.float_to_fp8(dec[fin], f), codes[fin])
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(50000) * 20).astype(np.float32)
    x = x[(np.abs(x) > 2.0 ** -5) & (np.abs(x) < 240)]  # normal range: round to nearest even, as torch
    for f in ("e4m3", "e4m3-sat"):
        assert np.array_equal(kv_oracle.float_to_fp8(x, f),
                              torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy())
    enc = lambda v, f="e4m3": int(kv_oracle.float_to_fp8(np.array([v], np.float32), f)[0])
    assert enc(1.0) == 0x38 and enc(240.0) == 0x77 and enc(-240.0) == 0xF7
    assert enc(np.inf) == 0x78 and enc(np.nan) == 0x79 and enc(-np.nan) == 0xF9
    assert enc(2.0 ** -9) == 0x01 and enc(-0.0) == 0x80 and enc(2.0 ** -11) == 0x00
    assert enc(250.0) == 0x78  # rounds past 240 in the normal path: +-Inf in every format
    # the reference's encoder code: 300 goes down the subnormal branch and keeps its low bits (0)
    assert enc(300.0) == 0x00 and enc(300.0, "e4m3-sat") == 0x78
    # a subnormal rounding up to the smallest normal: carry dropped (+0) / kept (0x08)
    assert enc(2.0 ** -6 * (1 - 2.0 ** -10)) == 0x00 and enc(2.0 ** -6 * (1 - 2.0 ** -10), "e4m3-sat") == 0x08
    # past the reference's defined range (negative shift count): +-Inf in every format
    assert enc(1e6) == 0x78 and enc(-1e6) == 0xF8 and enc(1e6, "e4m3-sat") == 0x78
    assert enc(57344.0, "e5m2") == 0x7B and enc(65536.0, "e5m2") == 0x7C and enc(65536.0, "e5m2-sat") == 0x7C


def test_fp8_codec_matches_reference_vectors():
    """kv_oracle's FP8 codec against the reference's own float8.metal functions,
    compiled as host C++ (tests/golden/make_fp8_golden.py): the decode of all
    256 codes, and the encode of every bfloat16 pattern, every float16 value
    and 2^17 seeded float32 patterns, bit for bit in both formats.  The "-sat"
    formats differ from the reference only on values past the last finite
    exponent and on subnormals that round up to the smallest normal."""
    import make_fp8_golden as g

    ref = np.load(os.path.join(ROOT, "tests", "golden", "fp8_ref.npz"))
    x = g.enc_inputs()
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(ref["enc_inputs_sha256"])
    f = x.view(np.float32)
    codes = np.arange(256, dtype=np.uint8)
    for fmt, finite_max, smallest_normal in (("e4m3", 240.0, 2.0 ** -6), ("e5m2", 57344.0, 2.0 ** -14)):
        got = kv_oracle.fp8_to_float(codes, fmt)
        want = ref[f"dec_{fmt}"].view(np.float32)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert np.array_equal(got[~np.isnan(got)].view(np.uint32), want[~np.isnan(want)].view(np.uint32))
        np.testing.assert_array_equal(kv_oracle.float_to_fp8(f, fmt), ref[f"enc_{fmt}"])
        sat = kv_oracle.float_to_fp8(f, fmt + "-sat")
        differ = sat != ref[f"enc_{fmt}"]
        a = np.abs(f[differ])
        assert ((a > finite_max) | (a < smallest_normal)).all()
        assert differ.any()


# ---- prefill / extend attention oracle --------------------------------------------

def test_prefill_mask_matches_make_mask():
    """offset_causal_mask is the mask PooledKVCache.make_mask returns (itself
    checked against the reference's make_mask tests in test_memory_pool.py),
    including the windowed case the reference pins (N=3, window 2)."""
    from sglang_mlx_b200.srt.mem_cache.memory_pool import PooledKVCache

    m = kv_oracle.offset_causal_mask(3, 3, 2)
    assert not m[2, 0] and m[2, 1] and m[2, 2]
    for prefix, n, w in [(0, 4, None), (3, 2, None), (5, 7, 3), (0, 9, 1), (10, 1, 4), (2, 6, 100)]:
        pc = PooledKVCache(None, 0)
        pc.set_indices(list(range(1, prefix + 1)), list(range(prefix + 1, prefix + n + 1)))
        want = np.asarray(pc.make_mask(N=n, return_array=True, window_size=w)) if n > 1 else None
        got = kv_oracle.offset_causal_mask(n, prefix + n, w)
        if want is not None:
            np.testing.assert_array_equal(got, want)
        assert got[-1, : prefix + n].sum() == (min(w, prefix + n) if w else prefix + n)


def test_sdpa_masked_against_torch():
    """The float64 masked SDPA against torch's scaled_dot_product_attention, an
    independent implementation of the same mathematics."""
    import torch

    rng = np.random.default_rng(61)
    for n, t, d, w in [(5, 5, 64, None), (7, 40, 128, None), (16, 300, 128, 33), (1, 9, 64, None)]:
        q = rng.standard_normal((n, d))
        k = rng.standard_normal((t, d))
        v = rng.standard_normal((t, d))
        mask = kv_oracle.offset_causal_mask(n, t, w)
        got = kv_oracle.sdpa_masked(q, k, v, d ** -0.5, mask)
        want = torch.nn.functional.scaled_dot_product_attention(
            torch.from_numpy(q)[None], torch.from_numpy(k)[None], torch.from_numpy(v)[None],
            attn_mask=torch.from_numpy(mask)[None], scale=d ** -0.5).numpy()[0]
        np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_prefill_oracle_layouts_agree_and_single_token_is_decode():
    """paged_prefill reads the paged layout, the flash layout and the token pool
    alike, and one new token per sequence is the decode oracle (whose softmax
    denominator carries the kernel's + 1e-6)."""
    import helpers

    lens = [7, 40, 100]
    c = cases.paged_batch(62, "float16", 3, 16, 4, 64, 16, lens)
    kc, vc = _fill(c)
    q = c["q"].astype(np.float64)  # [3, 16, 64]: one new token per sequence
    ind = np.arange(4, dtype=np.int32)
    lens32 = np.asarray(lens, np.int32)
    paged = kv_oracle.paged_prefill(q, kc, vc, c["block_tables"], ind, lens32, 4, c["scale"])
    dec = kv_oracle.paged_attention_v1(q, kc, vc, c["block_tables"], lens32, 4, c["scale"], 16, c["max_seq_len"])
    np.testing.assert_allclose(paged, dec, rtol=1e-5, atol=1e-6)
    for bs in (1, 16):
        fc = helpers.flash_case(62, "float16", 3, 16, 4, 64, bs, lens)
        fk, fv = helpers.oracle_flash_caches(fc)
        flash = kv_oracle.paged_prefill(fc["c"]["q"].astype(np.float64), fk, fv, fc["tables"], ind, lens32, 4,
                                        c["scale"])
        np.testing.assert_allclose(flash, paged, rtol=1e-12, atol=1e-12)
