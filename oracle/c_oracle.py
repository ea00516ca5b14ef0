"""ctypes loader of oracle/libkv_oracle.so (TEST INFRASTRUCTURE ONLY).

Builds the library on first use when a compiler is present; the GPU box uses
the prebuilt file shipped with the working tree.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libkv_oracle.so")
_lib = None

CODES = {"float32": 0, "float16": 1, "bfloat16": 2}


def build() -> str:
    src = os.path.join(_HERE, "kv_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        _lib = ctypes.CDLL(_SO)
        _lib.oracle_paged_attention.restype = ctypes.c_int
        _lib.oracle_paged_attention.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ]
        _lib.oracle_reshape_and_cache.restype = ctypes.c_int
        _lib.oracle_reshape_and_cache.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
        ]
        _lib.oracle_num_threads.restype = ctypes.c_int
    return _lib


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def paged_attention(query, q_dtype, key_cache, value_cache, cache_dtype, block_tables, context_lens, num_kv_heads,
                    scale, max_seq_len, alibi_slopes=None, seq_range=None, threads=0):
    """Float64 [B, Hq, D].  Arrays hold raw element storage: float32, float16,
    or uint16 bf16 bits (q_dtype / cache_dtype name the interpretation)."""
    q = np.ascontiguousarray(query)
    kc = np.ascontiguousarray(key_cache)
    vc = np.ascontiguousarray(value_cache)
    bt = np.ascontiguousarray(block_tables).astype(np.uint32, copy=False)
    cl = np.ascontiguousarray(context_lens).astype(np.uint32, copy=False)
    al = None if alibi_slopes is None else np.ascontiguousarray(alibi_slopes, dtype=np.float32)
    B, Hq, D = q.shape
    bs = vc.shape[3]
    out = np.zeros((B, Hq, D), dtype=np.float64)
    b0, b1 = seq_range if seq_range is not None else (0, B)
    rc = lib().oracle_paged_attention(_ptr(out), _ptr(q), CODES[q_dtype], _ptr(kc), _ptr(vc), CODES[cache_dtype],
                                      _ptr(bt), _ptr(cl), B, Hq, int(num_kv_heads), D, bs, bt.shape[1],
                                      int(max_seq_len), float(scale), _ptr(al), int(b0), int(b1), int(threads))
    if rc != 0:
        raise RuntimeError("oracle_paged_attention failed")
    return out


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping):
    """In-place vLLM-layout append on raw element storage (same dtype in and out)."""
    k = np.ascontiguousarray(key)
    v = np.ascontiguousarray(value)
    assert key_cache.flags.c_contiguous and value_cache.flags.c_contiguous
    sl = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    T, H, D = k.shape
    rc = lib().oracle_reshape_and_cache(_ptr(k), _ptr(v), _ptr(key_cache), _ptr(value_cache), _ptr(sl), T, H, D,
                                        value_cache.shape[3], key_cache.shape[4], k.itemsize, key_cache.shape[0])
    if rc != 0:
        raise RuntimeError("oracle_reshape_and_cache: slot beyond cache")
    return key_cache, value_cache
