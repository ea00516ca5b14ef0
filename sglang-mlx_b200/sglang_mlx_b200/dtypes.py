"""Element types understood by libkvcache and their DLPack / NumPy encodings.

bfloat16 has no NumPy dtype: device bf16 data is staged through NumPy as uint16
bit patterns, and float32 <-> bfloat16 conversion rounds to nearest even.
"""

from __future__ import annotations

import numpy as np

float32 = "float32"
float16 = "float16"
bfloat16 = "bfloat16"
int32 = "int32"
uint32 = "uint32"
int64 = "int64"
uint8 = "uint8"

# name -> (DLPack code, bits, itemsize, numpy storage dtype)
_TABLE = {
    float32: (2, 32, 4, np.dtype(np.float32)),
    float16: (2, 16, 2, np.dtype(np.float16)),
    bfloat16: (4, 16, 2, np.dtype(np.uint16)),
    int32: (0, 32, 4, np.dtype(np.int32)),
    uint32: (1, 32, 4, np.dtype(np.uint32)),
    int64: (0, 64, 8, np.dtype(np.int64)),
    uint8: (1, 8, 1, np.dtype(np.uint8)),
}
_FROM_DL = {(c, b): n for n, (c, b, _, _) in _TABLE.items()}


def canonical(dtype) -> str:
    """Accepts a dtype name, a NumPy dtype or a torch-like object with a name."""
    if isinstance(dtype, str):
        name = dtype.replace("torch.", "")
    else:
        try:
            name = np.dtype(dtype).name
        except TypeError:
            name = str(dtype).replace("torch.", "")
    aliases = {"half": float16, "float": float32, "bf16": bfloat16, "fp16": float16, "fp32": float32}
    name = aliases.get(name, name)
    if name not in _TABLE:
        raise ValueError(f"unsupported dtype {dtype!r}")
    return name


def itemsize(dtype) -> int:
    return _TABLE[canonical(dtype)][2]


def dl_code_bits(dtype) -> tuple[int, int]:
    c, b, _, _ = _TABLE[canonical(dtype)]
    return c, b


def from_dl(code: int, bits: int) -> str:
    try:
        return _FROM_DL[(code, bits)]
    except KeyError:
        raise ValueError(f"unsupported DLPack dtype code={code} bits={bits}") from None


def storage_dtype(dtype) -> np.dtype:
    return _TABLE[canonical(dtype)][3]


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN -> 0x7FC0)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = 0x7FC0
    return rounded


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)
