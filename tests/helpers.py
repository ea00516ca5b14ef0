"""Device-side helpers shared by the GPU tests: upload seeded cases, run the
CUDA path, download results."""

from __future__ import annotations

import numpy as np

import cases
from oracle import kv_oracle
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray

# north_star tolerance for fp16/bf16 attention outputs: 2e-3 abs / 1e-2 rel
ATOL_NS, RTOL_NS = 2e-3, 1e-2
# fp32 outputs (reference test tolerance is 5e-3 abs; fp32 math agrees far closer)
ATOL_F32, RTOL_F32 = 1e-4, 1e-4


def np_dtype_name(a: np.ndarray, hint: str | None = None) -> str:
    if hint is not None:
        return hint
    return {np.dtype(np.float16): "float16", np.dtype(np.float32): "float32"}[a.dtype]


def upload_case(c: dict, cache_dtype: str | None = None, q_dtype: str | None = None):
    """Uploads a case from tests/golden/cases.py.  bf16 cases carry float32 values."""
    dt = c.get("dtype")
    qd = q_dtype or (dt if dt else np_dtype_name(c["q"]))
    cd = cache_dtype or (dt if dt else np_dtype_name(c["k_cache"]))
    d = dict(
        q=DeviceArray.from_numpy(c["q"], dtype=qd),
        k=DeviceArray.from_numpy(c["k"], dtype=qd),
        v=DeviceArray.from_numpy(c["v"], dtype=qd),
        k_cache=DeviceArray.from_numpy(c["k_cache"], dtype=cd),
        v_cache=DeviceArray.from_numpy(c["v_cache"], dtype=cd),
        block_tables=DeviceArray.from_numpy(c["block_tables"]),
        context_lens=DeviceArray.from_numpy(c["context_lens"]),
        slot_mapping=DeviceArray.from_numpy(c["slot_mapping"]),
    )
    d["q_dtype"], d["cache_dtype"] = qd, cd
    return d


def fill_cache(d: dict):
    return mk.reshape_and_cache(d["k"], d["v"], d["k_cache"], d["v_cache"], d["slot_mapping"])


def oracle_fill(c: dict, cache_dtype: str):
    """The oracle's view of the filled caches (float32 values of the cache dtype)."""
    kc = c["k_cache"].astype(np.float32)
    vc = c["v_cache"].astype(np.float32)
    T = c["k"].shape[0]
    k = kv_oracle.round_to(c["k"], cache_dtype)
    v = kv_oracle.round_to(c["v"], cache_dtype)
    return kv_oracle.reshape_and_cache(k, v, kc, vc, c["slot_mapping"][:T])


def assert_close(got, ref, atol, rtol, what=""):
    ok, maxerr, excess = kv_oracle.allclose_report(got, ref, atol, rtol)
    assert ok, f"{what}: max |err| {maxerr:.3g}, worst excess over atol+rtol*|ref| {excess:.3g}"


def tolerance(out_dtype: str):
    return (ATOL_F32, RTOL_F32) if out_dtype == "float32" else (ATOL_NS, RTOL_NS)


def flash_case(seed, dtype, num_seqs, hq, hkv, d, bs, lens):
    """A batch in token-major caches.  bs = 1 gives a token pool: caches
    [slots, H, D] and block tables that are slot lists."""
    c = cases.paged_batch(seed, dtype, num_seqs, hq, hkv, d, 16, lens)
    nb16 = c["k_cache"].shape[0]
    slots = c["slot_mapping"].astype(np.int64)
    T = len(slots)
    if bs == 1:
        shape = (nb16 * 16 + 1, hkv, d)  # + the pool's padding slot 0
        slots = slots + 1
        t = np.arange(c["block_tables"].shape[1] * 16)
        tables = np.where(c["block_tables"][:, t // 16] >= 0, c["block_tables"][:, t // 16] * 16 + t % 16 + 1, 0)
    else:
        # re-block the same tokens into bs-token blocks of a permuted pool
        rng = np.random.default_rng(seed + 5)
        nbb = -(-nb16 * 16 // bs) + 2
        perm = rng.permutation(nbb)
        maxb = -(-c["block_tables"].shape[1] * 16 // bs)
        tables = np.full((num_seqs, maxb), -1, np.int64)
        pos = 0
        off = 0
        slots = np.empty(T, np.int64)
        for b, n in enumerate(c["context_lens"]):
            nb = -(-int(n) // bs)
            tables[b, :nb] = perm[pos:pos + nb]
            tt = np.arange(int(n))
            slots[off:off + n] = tables[b, tt // bs] * bs + tt % bs
            pos += nb
            off += int(n)
        shape = (nbb, bs, hkv, d)
    store = np.float16 if dtype == "float16" else np.float32
    return dict(c=c, shape=shape, tables=tables.astype(np.int32), slots=slots.astype(np.int32), bs=bs, store=store)


def upload_flash(fc):
    c = fc["c"]
    dt = c["dtype"]
    q = DeviceArray.from_numpy(c["q"], dtype=dt)
    k = DeviceArray.from_numpy(c["k"], dtype=dt)
    v = DeviceArray.from_numpy(c["v"], dtype=dt)
    kc = DeviceArray.zeros(fc["shape"], dt)
    vc = DeviceArray.zeros(fc["shape"], dt)
    mk.reshape_and_cache_flash(k, v, kc, vc, DeviceArray.from_numpy(fc["slots"]))
    return dict(q=q, kc=kc, vc=vc, tables=DeviceArray.from_numpy(fc["tables"]),
                lens=DeviceArray.from_numpy(c["context_lens"].astype(np.int32)))


def oracle_flash_caches(fc):
    """The oracle's view of the token-major caches upload_flash fills."""
    c = fc["c"]
    fk = np.zeros(fc["shape"], np.float32)
    fv = np.zeros(fc["shape"], np.float32)
    kv_oracle.reshape_and_cache_flash(kv_oracle.round_to(c["k"], c["dtype"]), kv_oracle.round_to(c["v"], c["dtype"]),
                                      fk, fv, fc["slots"])
    return fk, fv
