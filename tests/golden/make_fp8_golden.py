"""Generates tests/golden/fp8_ref.npz from the reference's own FP8 codec.

Run where the sglang-mlx checkout is present:
    python tests/golden/make_fp8_golden.py --reference PATH   (or SGLANG_MLX_REFERENCE=PATH)

It builds oracle/_ref/fp8_ref (`make -C oracle ref`): the codec functions of
paged_attention/metal/float8.metal:14-125, compiled unmodified from the
checkout as host C++ through oracle/msl_shim.h, and records
  * dec_e4m3 / dec_e5m2: the float32 bit pattern of every code 0..255
    (fp8_e4m3_to_float / fp8_e5m2_to_float, float8.metal:14-63);
  * enc_e4m3 / enc_e5m2: float_to_fp8_e4m3 / _e5m2 (float8.metal:65-125) of
    every bfloat16 bit pattern, every float16 value and a seeded sample of
    float32 bit patterns (enc_inputs_sha256 pins the regenerated inputs);
  * sweep_sha256_e4m3 / _e5m2: SHA-256 of the code of every float32 bit
    pattern 0 .. 2^32 - 1 in order (4 GiB per format, hashed as it streams).
Where the reference's encoder is undefined (a negative shift count past the
last finite exponent: |x| >= 2^14 for E4M3, |x| >= 2^16 for E5M2) the program
writes the saturated code +-Inf instead; every other input carries the
reference function's own result.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
SAMPLE_SEED = 8008
SAMPLE_N = 1 << 16


def enc_inputs() -> np.ndarray:
    """float32 bit patterns (uint32) fed to the encoders: every bfloat16
    pattern, every float16 value widened, then SAMPLE_N uniform random bit
    patterns and SAMPLE_N patterns with exponents near the FP8 ranges."""
    bf = (np.arange(1 << 16, dtype=np.uint32) << 16)
    f16 = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32).view(np.uint32)
    rng = np.random.default_rng(SAMPLE_SEED)
    uni = rng.integers(0, 1 << 32, size=SAMPLE_N, dtype=np.uint64).astype(np.uint32)
    exp = rng.integers(127 - 30, 127 + 20, size=SAMPLE_N, dtype=np.uint32)
    man = rng.integers(0, 1 << 23, size=SAMPLE_N, dtype=np.uint32)
    sgn = rng.integers(0, 2, size=SAMPLE_N, dtype=np.uint32)
    near = (sgn << 31) | (exp << 23) | man
    return np.concatenate([bf, f16, uni, near]).astype(np.uint32)


def run(binary: str, *args: str, stdin: bytes | None = None) -> bytes:
    return subprocess.run([binary, *args], input=stdin, stdout=subprocess.PIPE, check=True).stdout


def sweep_digest(binary: str, fmt: str) -> str:
    h = hashlib.sha256()
    with subprocess.Popen([binary, "sweep", fmt], stdout=subprocess.PIPE) as p:
        total = 0
        while True:
            chunk = p.stdout.read(1 << 24)
            if not chunk:
                break
            h.update(chunk)
            total += len(chunk)
        if p.wait() != 0 or total != 1 << 32:
            raise RuntimeError(f"sweep {fmt}: exit {p.returncode}, {total} bytes")
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SGLANG_MLX_REFERENCE"),
                    help="path of the sglang-mlx checkout (or set SGLANG_MLX_REFERENCE)")
    ap.add_argument("--out", default=os.path.join(HERE, "fp8_ref.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set SGLANG_MLX_REFERENCE to the sglang-mlx checkout")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REFERENCE={args.reference}"],
                   check=True)
    binary = os.path.join(ROOT, "oracle", "_ref", "fp8_ref")
    dec = np.frombuffer(run(binary, "dec"), np.uint32)
    x = enc_inputs()
    codes = np.frombuffer(run(binary, "enc", stdin=x.tobytes()), np.uint8).reshape(-1, 2)
    out = {
        "dec_e4m3": dec[:256].copy(),
        "dec_e5m2": dec[256:].copy(),
        "enc_e4m3": codes[:, 0].copy(),
        "enc_e5m2": codes[:, 1].copy(),
        "enc_inputs_sha256": np.array(hashlib.sha256(x.tobytes()).hexdigest()),
    }
    for fmt in ("e4m3", "e5m2"):
        print(f"sweep {fmt} ...", flush=True)
        out[f"sweep_sha256_{fmt}"] = np.array(sweep_digest(binary, fmt))
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} ({os.path.getsize(args.out) / 1e3:.0f} kB)")


if __name__ == "__main__":
    sys.exit(main())
