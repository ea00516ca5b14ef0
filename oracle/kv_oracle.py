"""CPU oracle of the paged-KV hot path (TEST INFRASTRUCTURE ONLY).

A NumPy restatement of sglang-mlx's reference algorithms, used by tests/,
__graft_entry__.smoke() and bench.py's CPU baseline as the checker.  The
product (libkvcache.so and its Python shim) never imports this package.

Pinned against the reference's own NumPy oracles
(tests/test_paged_attention_kernel.py:33-120, run on the reference's test
shapes and on config 1 by tests/golden/make_golden.py) and against the
reference MHATokenPool store/fetch run on a NumPy-backed mlx.core stand-in
(same script).  The fixtures live in tests/golden/.

Data formats (all NumPy; bf16 is carried as float32 values that are exactly
representable in bf16, or as uint16 bit patterns where marked):
  key_cache   [num_blocks, H, D/x, block_size, x]
  value_cache [num_blocks, H, D, block_size]
"""

from __future__ import annotations

import numpy as np


# ---------------------------------------------------------------------------
# element conversion (reshape_and_cache.metal:9-12: static_cast, i.e. round to
# nearest even when narrowing)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = 0x7FC0  # utils.metal:23-26
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Values of `a` rounded to `dtype` ('float32'|'float16'|'bfloat16'), returned as float32."""
    if dtype == "float32":
        return np.asarray(a, dtype=np.float32)
    if dtype == "float16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(a))
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# reshape_and_cache — reshape_and_cache.metal:35-69
# ---------------------------------------------------------------------------
def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping):
    """In-place scatter of key/value [T, H, D] into the vLLM-layout caches.

    slot < 0 skips the token (:36-39); block = slot // bs, offset = slot % bs
    (:41-42); K[block, h, d // x, offset, d % x] = key[t, h, d] (:54-59);
    V[block, h, d, offset] = value[t, h, d] (:61-65).  Element conversion is the
    caller's job (pass key/value already in the cache dtype).
    """
    slots = np.asarray(slot_mapping).astype(np.int64)
    keep = slots >= 0
    if not keep.any():
        return key_cache, value_cache
    s = slots[keep]
    k = np.asarray(key)[keep]
    v = np.asarray(value)[keep]
    T, H, D = k.shape
    bs = value_cache.shape[3]
    x = key_cache.shape[4]
    blk, off = s // bs, s % bs
    # K: [T, H, D] -> [T, H, D/x, x]
    kc = k.reshape(T, H, D // x, x)
    key_cache[blk[:, None, None], np.arange(H)[None, :, None], np.arange(D // x)[None, None, :], off[:, None, None], :] = kc
    value_cache[blk[:, None, None], np.arange(H)[None, :, None], np.arange(D)[None, None, :], off[:, None, None]] = v
    return key_cache, value_cache


# ---------------------------------------------------------------------------
# reshape_and_cache_flash — reshape_and_cache.metal:115-136
# ---------------------------------------------------------------------------
def reshape_and_cache_flash(key, value, key_cache, value_cache, slot_mapping):
    """Caches [nb, bs, H, D] (or the pool's [slots, H, D]); row copy at slot."""
    slots = np.asarray(slot_mapping).astype(np.int64)
    keep = slots >= 0
    kflat = key_cache.reshape(-1, *key_cache.shape[-2:])
    vflat = value_cache.reshape(-1, *value_cache.shape[-2:])
    kflat[slots[keep]] = np.asarray(key)[keep]
    vflat[slots[keep]] = np.asarray(value)[keep]
    return key_cache, value_cache


# ---------------------------------------------------------------------------
# MHATokenPool.store / fetch — memory_pool.py:117-159
# ---------------------------------------------------------------------------
def pool_store(k_buffer, v_buffer, indices, keys, values):
    """keys/values (1, H, S, D) -> transpose to (S, H, D) -> scatter at indices."""
    idx = np.asarray(indices, dtype=np.int64)
    k_buffer[idx] = np.transpose(np.asarray(keys)[0], (1, 0, 2))
    v_buffer[idx] = np.transpose(np.asarray(values)[0], (1, 0, 2))


def pool_fetch(k_buffer, v_buffer, indices):
    """Gather (T, H, D) at indices -> transpose -> (1, H, T, D)."""
    idx = np.asarray(indices, dtype=np.int64)
    k = np.transpose(k_buffer[idx], (1, 0, 2))[None]
    v = np.transpose(v_buffer[idx], (1, 0, 2))[None]
    return k, v


# ---------------------------------------------------------------------------
# FP8 codecs — float8.metal:13-125 (used by convert_fp8.metal:13-80)
# ---------------------------------------------------------------------------
FP8_FORMATS = ("e4m3", "e5m2", "e4m3-sat", "e5m2-sat")


def _fp8_layout(fmt: str):
    """(exponent bits, mantissa bits, bias, saturating) of an FP8 format name."""
    if fmt not in FP8_FORMATS:
        raise ValueError(f"unknown FP8 format {fmt!r}")
    eb, mb, bias = (4, 3, 7) if fmt.startswith("e4m3") else (5, 2, 15)
    return eb, mb, bias, fmt.endswith("-sat")


def fp8_to_float(v, fmt: str = "e4m3"):
    """Decodes uint8 codes (float8.metal:14-63).  Both formats keep the
    all-ones exponent for Inf (mantissa 0) and NaN, IEEE style: E4M3's largest
    finite value is 240 here, not OCP E4M3FN's 448.  The "-sat" formats decode
    the same way."""
    eb, mb, bias, _ = _fp8_layout(fmt)
    v = np.asarray(v, dtype=np.uint8).astype(np.int64)
    s = v >> 7
    e = (v >> mb) & ((1 << eb) - 1)
    m = v & ((1 << mb) - 1)
    sub = np.ldexp(m / float(1 << mb), 1 - bias)
    nor = np.ldexp(1.0 + m / float(1 << mb), e - bias)
    out = np.where(e == 0, sub, nor)
    top = e == (1 << eb) - 1
    out = np.where(top, np.where(m == 0, np.inf, np.nan), out)
    return np.where(s == 1, -out, out).astype(np.float32)


def float_to_fp8(f, fmt: str = "e4m3"):
    """Encodes float32 values as float8.metal:69-118 (detail::fp32_to_fp8)
    does, step for step:
      * NaN keeps its sign with mantissa 1, +-Inf the all-ones exponent (:75-79);
      * biased FP8 exponent in [1, last finite]: round to nearest even, a
        mantissa carry past the last finite exponent gives +-Inf (:85-103);
      * below 2^(1 - bias - mantissa bits): +-0 (:106-107);
      * otherwise the subnormal branch (:110-116): the mantissa with its
        implicit 1 shifted right by (1 - e) + (23 - mantissa bits), rounded half
        up, of which only the mantissa bits are kept.  So a subnormal that rounds
        up to the smallest normal becomes +-0, and values past the last finite
        exponent (E4M3: 256 <= |x| < 2^14) get the low bits of that shift ("300
        encodes as 0").
    Past that (E4M3 |x| >= 2^14, E5M2 |x| >= 2^16) the reference's shift count is
    negative, undefined in C++ and MSL; there the result is +-Inf.
    The "-sat" formats keep the encoder's stated behaviour (:65-68) instead:
    +-Inf for every value past the last finite exponent, and a subnormal that
    rounds up keeps its carry into the smallest normal."""
    eb, mb, bias, sat = _fp8_layout(fmt)
    bits = np.ascontiguousarray(np.asarray(f, dtype=np.float32)).view(np.uint32).astype(np.int64)
    s = bits >> 31
    a = bits & 0x7FFFFFFF
    top = ((1 << eb) - 1) << mb
    e = ((a >> 23) & 0xFF) - 127
    m = a & 0x7FFFFF
    exp_max = (1 << eb) - 2
    ef = e + bias
    shift = 23 - mb
    mant = m >> shift
    lsb = mant & 1
    rnd = (m >> (shift - 1)) & 1
    sticky = (m & ((1 << (shift - 1)) - 1)) != 0
    mant = mant + (rnd & (sticky | lsb))
    carry = (mant >> mb) != 0
    ef_n = np.where(carry, ef + 1, ef)
    mant = np.where(carry, 0, mant)
    normal = np.where(ef_n > exp_max, (s << 7) | top, (s << 7) | (ef_n << mb) | (mant & ((1 << mb) - 1)))
    rshift = (1 - ef) + (23 - mb)
    rounded = ((0x800000 | m) + (np.int64(1) << np.clip(rshift - 1, 0, 62))) >> np.clip(rshift, 0, 62)
    if sat:
        branch = (s << 7) | rounded  # rounded <= 1 << mb: the carry lands in the exponent field
        past = ef > exp_max
    else:
        branch = (s << 7) | (rounded & ((1 << mb) - 1))
        past = rshift < 1
    sub = np.where(ef < 1 - mb, s << 7, np.where(past, (s << 7) | top, branch))
    out = np.where((ef >= 1) & (ef <= exp_max), normal, sub)
    nan_inf = a >= 0x7F800000
    out = np.where(nan_inf, (s << 7) | top | (a != 0x7F800000), out)
    return out.astype(np.uint8)


def quantize(x, scale: float, fmt: str = "e4m3"):
    """Higher precision -> FP8: encode(x / scale) (convert_fp8.metal:33-36)."""
    return float_to_fp8(np.asarray(x, dtype=np.float32) / np.float32(scale), fmt)


def dequantize(q, scale: float, fmt: str = "e4m3"):
    """FP8 -> float: decode(q) * scale (convert_fp8.metal:28-31)."""
    return fp8_to_float(q, fmt) * np.float32(scale)


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale, fmt="e4m3"):
    """Quantising append into uint8 caches of the vLLM layout with x = 16 (the
    index math of reshape_and_cache.metal:41-65 on quantize(x, scale) codes)."""
    kq = quantize(np.asarray(key, dtype=np.float32), k_scale, fmt)
    vq = quantize(np.asarray(value, dtype=np.float32), v_scale, fmt)
    return reshape_and_cache(kq, vq, key_cache, value_cache, slot_mapping)


def paged_attention_fp8(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale, block_size,
                        max_seq_len, k_scale, v_scale, fmt="e4m3", alibi_slopes=None):
    """paged_attention_v1 (float64) over the dequantised one-byte caches."""
    kc = dequantize(key_cache, k_scale, fmt)
    vc = dequantize(value_cache, v_scale, fmt)
    return paged_attention_v1(query, kc, vc, block_tables, context_lens, num_kv_heads, scale, block_size,
                              max_seq_len, alibi_slopes)


# ---------------------------------------------------------------------------
# copy_blocks / swap_blocks — copy_blocks.metal:9-75 (host: mlx_cache.cpp:302-370)
# ---------------------------------------------------------------------------
def copy_blocks(key_caches, value_caches, block_mapping):
    """In place, for every layer and pair (src, dst): block dst of the key and
    value caches := block src (a block is everything behind the leading index,
    copy_blocks.metal:21-43).  Pairs are applied in order; the kernel runs them
    in parallel, which agrees whenever no block is both read and written."""
    pairs = np.asarray(block_mapping, dtype=np.int64).reshape(-1, 2)
    for kc, vc in zip(key_caches, value_caches):
        for s, d in pairs:
            kc[d] = kc[s]
            vc[d] = vc[s]
    return key_caches, value_caches


def swap_blocks(src, dst, block_mapping):
    """dst[d] := src[s] for every pair (copy_blocks.metal:60-75); returns dst."""
    for s, d in np.asarray(block_mapping, dtype=np.int64).reshape(-1, 2):
        dst[d] = src[s]
    return dst


# ---------------------------------------------------------------------------
# paged attention decode — paged_attention_kernels.metal:37-168
# ---------------------------------------------------------------------------
def gather_seq(key_cache, value_cache, block_table, n_tokens, kv_head):
    """(n_tokens, D) K and V of one sequence and KV head, through its block table."""
    bs = value_cache.shape[3]
    x = key_cache.shape[4]
    nb = -(-n_tokens // bs)
    blocks = np.asarray(block_table[:nb]).astype(np.uint32).astype(np.int64)
    # K page [D/x, bs, x] -> [bs, D]
    kp = key_cache[blocks, kv_head]                     # [nb, D/x, bs, x]
    k = np.transpose(kp, (0, 2, 1, 3)).reshape(nb * bs, -1)[:n_tokens]
    vp = value_cache[blocks, kv_head]                   # [nb, D, bs]
    v = np.transpose(vp, (0, 2, 1)).reshape(nb * bs, -1)[:n_tokens]
    return k, v


def attend(q, k, v, scale, alibi_slope=0.0, context_len=None):
    """softmax(scale * k @ q (+ alibi)) @ v in float64, denominator sum + 1e-6.

    q [G, D], k/v [T, D].  Mirrors paged_attention_kernels.metal:88-97 (logits),
    :104-144 (max-subtracted softmax, inv_sum = 1 / (sum + 1e-6)) and :146-168.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    T = k.shape[0]
    logits = (q @ k.T) * float(scale)                  # [G, T]
    if context_len is None:
        context_len = T
    slope = np.broadcast_to(np.asarray(alibi_slope, dtype=np.float64), (q.shape[0],))
    if np.any(slope != 0):
        pos = np.arange(T, dtype=np.float64) - context_len + 1
        logits = logits + slope[:, None] * pos[None, :]
    m = logits.max(axis=1, keepdims=True)
    p = np.exp(logits - m)
    return (p @ v) / (p.sum(axis=1, keepdims=True) + 1e-6)


def paged_attention_v1(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                       block_size, max_seq_len, alibi_slopes=None):
    """Float64 result [B, Hq, D] of paged_attention_v1 (not rounded).

    context_len == 0 or > max_seq_len -> zeros (:45-50); kv_head = h // G (:57-58);
    block tables / context lens read as uint32 (:22-23).
    """
    q = np.asarray(query, dtype=np.float64)
    B, Hq, D = q.shape
    G = Hq // num_kv_heads
    out = np.zeros((B, Hq, D), dtype=np.float64)
    lens = np.asarray(context_lens).astype(np.uint32)
    for b in range(B):
        C = int(lens[b])
        if C == 0 or C > max_seq_len:
            continue
        for kvh in range(num_kv_heads):
            k, v = gather_seq(key_cache, value_cache, block_tables[b], C, kvh)
            hs = slice(kvh * G, (kvh + 1) * G)
            slope = 0.0 if alibi_slopes is None else np.asarray(alibi_slopes, dtype=np.float64)[hs]
            out[b, hs] = attend(q[b, hs], k, v, scale, slope, C)
    return out


def gather_seq_flash(key_cache, value_cache, block_table, n_tokens, kv_head):
    """(n_tokens, D) K and V of one sequence and KV head from token-major caches:
    [nb, bs, H, D] (reshape_and_cache.metal:115-136 layout) or the pool's
    [slots, H, D] (memory_pool.py:102-108), where the table row is the slot list."""
    if key_cache.ndim == 3:
        key_cache = key_cache[:, None]
        value_cache = value_cache[:, None]
    bs = key_cache.shape[1]
    t = np.arange(n_tokens)
    blocks = np.asarray(block_table).astype(np.uint32).astype(np.int64)[t // bs]
    return key_cache[blocks, t % bs, kv_head], value_cache[blocks, t % bs, kv_head]


def paged_attention_flash(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                          max_seq_len, alibi_slopes=None):
    """paged_attention_v1's result over token-major caches (same edge rules:
    zeros when context_len == 0 or > max_seq_len; kv_head = h // G)."""
    q = np.asarray(query, dtype=np.float64)
    B, Hq, D = q.shape
    G = Hq // num_kv_heads
    out = np.zeros((B, Hq, D), dtype=np.float64)
    lens = np.asarray(context_lens).astype(np.uint32)
    for b in range(B):
        C = int(lens[b])
        if C == 0 or C > max_seq_len:
            continue
        for kvh in range(num_kv_heads):
            k, v = gather_seq_flash(key_cache, value_cache, block_tables[b], C, kvh)
            hs = slice(kvh * G, (kvh + 1) * G)
            slope = 0.0 if alibi_slopes is None else np.asarray(alibi_slopes, dtype=np.float64)[hs]
            out[b, hs] = attend(q[b, hs], k, v, scale, slope, C)
    return out


def paged_attention_splitk(query, key_cache, value_cache, block_tables, context_lens, num_kv_heads, scale,
                           block_size, max_seq_len, partition_size, alibi_slopes=None):
    """Split-K restatement: per partition (m_p, l_p, o_p), merged with LSE weights.

    Returns (out [B, Hq, D], partial maxima, partial sums) in float64.  The
    merge is out = sum_p e^{m_p - M} o_p / (sum_p e^{m_p - M} l_p + 1e-6).
    """
    q = np.asarray(query, dtype=np.float64)
    B, Hq, D = q.shape
    G = Hq // num_kv_heads
    P = -(-max_seq_len // partition_size)
    out = np.zeros((B, Hq, D))
    pm = np.full((B, Hq, P), -np.inf)
    pl = np.zeros((B, Hq, P))
    lens = np.asarray(context_lens).astype(np.uint32)
    for b in range(B):
        C = int(lens[b])
        if C == 0 or C > max_seq_len:
            continue
        for kvh in range(num_kv_heads):
            k, v = gather_seq(key_cache, value_cache, block_tables[b], C, kvh)
            hs = slice(kvh * G, (kvh + 1) * G)
            qq = q[b, hs]
            logits = (qq @ np.asarray(k, np.float64).T) * float(scale)
            if alibi_slopes is not None:
                sl = np.asarray(alibi_slopes, dtype=np.float64)[hs]
                logits = logits + sl[:, None] * (np.arange(C) - C + 1)[None, :]
            acc = np.zeros((G, D))
            nparts = -(-C // partition_size)
            ms = np.empty((G, nparts))
            ls = np.empty((G, nparts))
            os_ = np.empty((nparts, G, D))
            for p in range(nparts):
                seg = slice(p * partition_size, min(C, (p + 1) * partition_size))
                lg = logits[:, seg]
                m = lg.max(axis=1)
                e = np.exp(lg - m[:, None])
                ms[:, p], ls[:, p] = m, e.sum(axis=1)
                os_[p] = e @ np.asarray(v[seg], np.float64)
            M = ms.max(axis=1)
            w = np.exp(ms - M[:, None])
            L = (w * ls).sum(axis=1)
            acc = np.einsum("gp,pgd->gd", w, os_)
            out[b, hs] = acc / (L[:, None] + 1e-6)
            pm[b, hs, :nparts] = ms
            pl[b, hs, :nparts] = ls
    return out, pm, pl


# ---------------------------------------------------------------------------
# gather + SDPA dataflow of the reference's serving path (memory_pool.py:139-159
# then mx.fast.scaled_dot_product_attention; bench_paged_vs_gather.py:83-103)
# ---------------------------------------------------------------------------
def gather_sdpa(query, k_contig, v_contig, scale):
    """query [B, Hq, D]; k/v (1, Hkv, T, D) gathered; GQA broadcast.  Float64."""
    q = np.asarray(query, dtype=np.float64)
    B, Hq, D = q.shape
    Hkv = k_contig.shape[1]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D))
    for h in range(Hkv):
        k = np.asarray(k_contig[0, h], np.float64)
        v = np.asarray(v_contig[0, h], np.float64)
        out[:, h * G:(h + 1) * G] = attend(q[:, h * G:(h + 1) * G].reshape(-1, D), k, v, scale).reshape(B, G, D)
    return out


# ---------------------------------------------------------------------------
# prefill / extend attention (the reference runs it as mlx SDPA over the K/V
# that PooledKVCache.update_and_fetch gathers, memory_pool.py:205-234, under
# the mask of PooledKVCache.make_mask, memory_pool.py:240-270)
# ---------------------------------------------------------------------------
def offset_causal_mask(n_new, kv_len, window=None):
    """Boolean [n_new, kv_len]: new token t (cache position prefix + t, prefix =
    kv_len - n_new) sees cache token j iff j <= prefix + t and, with a window w,
    j > prefix + t - w.  This is what mlx-lm's create_attention_mask(N, offset,
    window_size) means for make_mask: "causal" with the offset, and the
    windowed boolean mask the reference pins in tests/test_memory_pool.py:
    291-320 (N=3, window 2: token 2 sees 1 and 2, not 0)."""
    prefix = kv_len - n_new
    pos = prefix + np.arange(n_new)[:, None]
    j = np.arange(kv_len)[None, :]
    m = j <= pos
    if window:
        m &= j > pos - window
    return m


def sdpa_masked(q, k, v, scale, mask):
    """softmax(scale * q @ k^T, masked) @ v in float64, no epsilon (mlx SDPA);
    a row with no visible key is 0.  q [N, D], k/v [T, D], mask [N, T]."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    logits = np.where(mask, (q @ k.T) * float(scale), -np.inf)
    m = logits.max(axis=1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(logits - m)
    s = p.sum(axis=1, keepdims=True)
    return np.where(s > 0, (p @ v) / np.where(s > 0, s, 1.0), 0.0)


def paged_prefill(query, key_cache, value_cache, block_tables, qo_indptr, kv_lens, num_kv_heads, scale,
                  window=None):
    """Float64 [num_tokens, Hq, D] of prefill / extend attention: sequence b's new
    tokens (rows qo_indptr[b] .. qo_indptr[b+1]-1) attend to its kv_lens[b]
    cache tokens under offset_causal_mask; GQA as the decode (kv head h // G).
    Caches in the paged layout (5-D key cache) or token-major ([nb, bs, H, D] /
    the pool's [slots, H, D])."""
    q = np.asarray(query, dtype=np.float64)
    T, Hq, D = q.shape
    G = Hq // num_kv_heads
    out = np.zeros((T, Hq, D))
    ind = np.asarray(qo_indptr).astype(np.int64)
    lens = np.asarray(kv_lens).astype(np.int64)
    for b in range(len(lens)):
        q0, q1, kvl = int(ind[b]), int(ind[b + 1]), int(lens[b])
        if q1 <= q0:
            continue
        mask = offset_causal_mask(q1 - q0, kvl, window)
        for h in range(num_kv_heads):
            if key_cache.ndim == 5:
                k, v = gather_seq(key_cache, value_cache, block_tables[b], kvl, h)
            else:
                k, v = gather_seq_flash(key_cache, value_cache, block_tables[b], kvl, h)
            for g in range(G):
                out[q0:q1, h * G + g] = sdpa_masked(q[q0:q1, h * G + g], k, v, scale, mask)
    return out


def allclose_report(got, ref, atol, rtol):
    """(ok, max_abs_err, worst_excess) for |got - ref| <= atol + rtol * |ref|."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    excess = float(np.max(err - bound)) if err.size else 0.0
    return bool(np.all(err <= bound)), float(err.max() if err.size else 0.0), excess
