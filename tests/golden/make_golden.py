"""Generates tests/golden/golden.npz from the reference implementation itself.

Run in a container where the reference checkout is present:
    python tests/golden/make_golden.py --reference PATH   (or SGLANG_MLX_REFERENCE=PATH)

What it runs (all reference code, unmodified, imported from the checkout):
  * `ref_reshape_and_cache` and `ref_paged_attention`, the NumPy oracles of
    tests/test_paged_attention_kernel.py:33-120, on the reference tests' own
    shapes (cases.ref_*) and on BASELINE.json config 1 (fp16, and a bf16-valued
    variant);
  * `TokenPoolAllocator` and `MHATokenPool` of
    sglang_mlx/srt/mem_cache/memory_pool.py, with `mlx.core` replaced by a
    NumPy-backed stand-in (mx.array/zeros/transpose/expand_dims map to NumPy),
    on a scripted store/fetch/alloc/free sequence.
MLX itself is not installed, so `mx.fast.scaled_dot_product_attention` cannot
be run; the kernel-level oracle above is the pin.  Large arrays are stored as
SHA-256 digests of their bytes; small ones verbatim.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def install_numpy_mlx() -> None:
    """A NumPy-backed `mlx.core` with the names the reference's pool and test
    modules touch at import time and in the code paths run here."""
    core = types.ModuleType("mlx.core")
    core.array = lambda a, dtype=None: np.array(a, dtype=dtype)
    core.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype)
    core.transpose = lambda a, axes=None: np.transpose(a, axes)
    core.expand_dims = lambda a, axis: np.expand_dims(a, axis)
    core.float16, core.float32, core.int32, core.uint32 = np.float16, np.float32, np.int32, np.uint32
    core.bfloat16 = np.float32
    core.Dtype = type
    pkg = types.ModuleType("mlx")
    pkg.core = core
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = core


def load_reference(ref: str):
    install_numpy_mlx()
    sys.path.insert(0, ref)
    spec = importlib.util.spec_from_file_location("ref_kernel_tests", os.path.join(ref, "tests",
                                                                                   "test_paged_attention_kernel.py"))
    kt = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(kt)
    from sglang_mlx.srt.mem_cache import memory_pool as mp
    return kt, mp


def run_kernel_case(kt, name: str, c: dict, out: dict, store_caches: bool) -> None:
    t0 = time.time()
    kc = c["k_cache"].copy()
    vc = c["v_cache"].copy()
    # The reference fixture hands float32 K/V to an fp16 cache; the Metal kernel
    # converts element-wise (static_cast, round to nearest even) and NumPy's
    # assignment into the fp16 array does the same.
    ref_k, ref_v = kt.ref_reshape_and_cache(c["k"], c["v"], kc, vc, c["slot_mapping"])
    attn = kt.ref_paged_attention(c["q"], ref_k, ref_v, c["block_tables"], c["context_lens"], c["scale"],
                                  c["num_kv_heads"])
    out[f"{name}/inputs_sha"] = np.array(cases.digest(c["q"], c["k"], c["v"], c["block_tables"],
                                                      c["context_lens"], c["slot_mapping"]))
    out[f"{name}/k_cache_sha"] = np.array(cases.digest(ref_k))
    out[f"{name}/v_cache_sha"] = np.array(cases.digest(ref_v))
    if store_caches:
        out[f"{name}/k_cache"] = ref_k
        out[f"{name}/v_cache"] = ref_v
    out[f"{name}/attn"] = attn
    print(f"  {name}: attn {attn.shape} {attn.dtype} in {time.time() - t0:.1f}s", flush=True)


def run_pool_case(mp, out: dict) -> None:
    """Scripted allocator + MHATokenPool run (memory_pool.py:27-159)."""
    rng = np.random.default_rng(123)
    alloc = mp.TokenPoolAllocator(pool_size=40)
    a1 = alloc.alloc(5)
    a2 = alloc.alloc(7)
    alloc.free(a1[1:3])
    a3 = alloc.alloc(4)
    out["pool/alloc_seq"] = np.array(a1 + [-1] + a2 + [-1] + a3, dtype=np.int64)
    out["pool/available"] = np.array(alloc.available_size)

    pool = mp.MHATokenPool(pool_size=40, num_layers=2, n_kv_heads=4, head_dim=8, dtype=np.float32)
    writes = []
    for layer, idx in ((0, a2), (1, a3), (0, a3[:2]), (0, [5, 10, 20])):
        S = len(idx)
        k = rng.standard_normal((1, 4, S, 8), dtype=np.float32)
        v = rng.standard_normal((1, 4, S, 8), dtype=np.float32)
        pool.store(layer, list(idx), k, v)
        writes.append((layer, list(idx), k, v))
    for i, (layer, idx, k, v) in enumerate(writes):
        out[f"pool/write{i}/layer"] = np.array(layer)
        out[f"pool/write{i}/idx"] = np.array(idx, dtype=np.int64)
        out[f"pool/write{i}/k"] = k
        out[f"pool/write{i}/v"] = v
    fetch_idx = [a2[3], a3[0], 5, 20, a2[0], 10, 0]
    for layer in (0, 1):
        kf, vf = pool.fetch(layer, fetch_idx)
        out[f"pool/fetch{layer}/k"] = np.asarray(kf)
        out[f"pool/fetch{layer}/v"] = np.asarray(vf)
    out["pool/fetch_idx"] = np.array(fetch_idx, dtype=np.int64)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SGLANG_MLX_REFERENCE"),
                    help="path of the sglang-mlx checkout (or set SGLANG_MLX_REFERENCE)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set SGLANG_MLX_REFERENCE to the sglang-mlx checkout")
    kt, mp = load_reference(args.reference)
    out: dict = {}
    print("reference kernel oracles:", flush=True)
    run_kernel_case(kt, "ref_setup", cases.ref_setup_data(), out, store_caches=True)
    for hd in (32, 128):
        for bs in (8, 16):
            run_kernel_case(kt, f"ref_various_{hd}_{bs}", cases.ref_various(hd, bs), out, store_caches=True)
    run_kernel_case(kt, "ref_legacy_2048", cases.ref_legacy_2048(), out, store_caches=True)
    run_kernel_case(kt, "config1_fp16", cases.config1(dtype="float16"), out, store_caches=False)
    run_kernel_case(kt, "config1_bf16", cases.config1(seed=12, dtype="bfloat16"), out, store_caches=False)
    print("reference pool:", flush=True)
    run_pool_case(mp, out)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} ({os.path.getsize(args.out) / 1e3:.0f} kB)")


if __name__ == "__main__":
    main()
