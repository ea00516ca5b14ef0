"""ctypes binding of libkvcache.so (the C ABI declared in include/kvcache.h).

The shared library is built in-tree next to this file.  There is no fallback:
importing this module without the library raises ImportError, so a missing
build can never silently turn into a CPU path.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KVC_LIBRARY", os.path.join(_HERE, "libkvcache.so"))

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"libkvcache.so not found at {LIB_PATH}; build it with "
        "`make -C sglang-mlx_b200/csrc` (or __graft_entry__.build())"
    )

lib = ctypes.CDLL(LIB_PATH)

KVC_OK = 0
KVC_EINVAL = 1
KVC_ECUDA = 2
KVC_ENOMEM = 3
KVC_EUNSUPPORTED = 4

STATUS_SLOT_OOB = 0x1
STATUS_BLOCK_OOB = 0x2
STATUS_WAIT_TIMEOUT = 0x4
STATUS_INDEX_OOB = 0x8
STATUS_PREFIX_MISMATCH = 0x10
STATUS_PLAN_MISMATCH = 0x20

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes).  Every symbol of include/kvcache.h.
SIGNATURES: dict[str, tuple] = {
    "kvc_last_error": (ctypes.c_char_p, []),
    "kvc_version": (ctypes.c_char_p, []),
    "kvc_get_status": (_i, [_i, ctypes.POINTER(ctypes.c_uint32), _i]),
    "kvc_paged_attention_v1": (_i, [_p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _p]),
    "kvc_paged_attention_v2": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _p],
    ),
    "kvc_paged_attention_v2_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _p]),
    "kvc_decode_plan_size": (ctypes.c_int64, [_i, _i, _i, _i]),
    "kvc_decode_plan": (_i, [_p, _p, _i, _i, _i, _p]),
    "kvc_paged_attention_planned": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _p, _p],
    ),
    "kvc_paged_attention_planned_append": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _p, _p],
    ),
    "kvc_paged_attention_cascade": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _i, _i, _p],
    ),
    "kvc_paged_prefill": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _i, _p]),
    "kvc_paged_attention_flash": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _i, _p],
    ),
    "kvc_reshape_and_cache": (_i, [_p, _p, _p, _p, _p, _p]),
    "kvc_reshape_and_cache_flash": (_i, [_p, _p, _p, _p, _p, _p]),
    "kvc_gather_kv": (_i, [_p, _p, _p, _p, _p, _p]),
    "kvc_copy_blocks": (_i, [_p, _i, _p, _i, _p, _p]),
    "kvc_reshape_and_cache_fp8": (_i, [_p, _p, _p, _p, _p, _f, _f, _i, _p]),
    "kvc_paged_attention_fp8": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _f, _f, _i, _i, _p],
    ),
    "kvc_paged_attention_fp8_planned": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _f, _i, _i, _p, _f, _f, _i, _i, _p, _p],
    ),
    "kvc_convert_fp8": (_i, [_p, _p, _f, _i, _p]),
    "kvc_swap_blocks": (_i, [_p, _p, _p, _p]),
    "kvc_get_max_shared_memory_per_block_device_attribute": (
        _i,
        [_i, ctypes.POINTER(ctypes.c_int64)],
    ),
    "kvc_get_device_attribute": (_i, [_i, _i, ctypes.POINTER(ctypes.c_int64)]),
    "kvc_device_count": (_i, [ctypes.POINTER(_i)]),
    "kvc_set_device": (_i, [_i]),
    "kvc_get_device": (_i, [ctypes.POINTER(_i)]),
    "kvc_malloc": (_i, [ctypes.POINTER(_p), _sz]),
    "kvc_free": (_i, [_p]),
    "kvc_malloc_host": (_i, [ctypes.POINTER(_p), _sz]),
    "kvc_free_host": (_i, [_p]),
    "kvc_memcpy_async": (_i, [_p, _p, _sz, _i, _p]),
    "kvc_memset_async": (_i, [_p, _i, _sz, _p]),
    "kvc_stream_create": (_i, [ctypes.POINTER(_p)]),
    "kvc_stream_destroy": (_i, [_p]),
    "kvc_stream_synchronize": (_i, [_p]),
    "kvc_device_synchronize": (_i, []),
    "kvc_event_create": (_i, [ctypes.POINTER(_p)]),
    "kvc_event_destroy": (_i, [_p]),
    "kvc_event_record": (_i, [_p, _p]),
    "kvc_stream_wait_event": (_i, [_p, _p]),
    "kvc_event_synchronize": (_i, [_p]),
    "kvc_event_elapsed_ms": (_i, [_p, _p, ctypes.POINTER(_f)]),
    "kvc_l2_flush": (_i, [_p, _sz, _p]),
    "kvc_stream_begin_capture": (_i, [_p]),
    "kvc_stream_end_capture": (_i, [_p, ctypes.POINTER(_p)]),
    "kvc_graph_launch": (_i, [_p, _p]),
    "kvc_graph_destroy": (_i, [_p]),
    "kvc_launch_count": (ctypes.c_uint64, []),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class KVCacheError(RuntimeError):
    """A CUDA-side failure reported by libkvcache."""


def last_error() -> str:
    msg = lib.kvc_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    """Raises the Python exception matching a libkvcache status code.

    Argument errors map to ValueError with the reference's message text (the
    nanobind binding turns std::invalid_argument into ValueError).
    """
    if rc == KVC_OK:
        return
    msg = last_error()
    if rc == KVC_EINVAL:
        raise ValueError(msg)
    if rc == KVC_ENOMEM:
        raise MemoryError(msg)
    if rc == KVC_EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise KVCacheError(msg)


def launch_count() -> int:
    return int(lib.kvc_launch_count())


def device_count() -> int:
    n = ctypes.c_int(0)
    rc = lib.kvc_device_count(ctypes.byref(n))
    return n.value if rc == KVC_OK else 0


def set_device(device: int) -> None:
    check(lib.kvc_set_device(int(device)))


def current_device() -> int:
    d = ctypes.c_int(0)
    check(lib.kvc_get_device(ctypes.byref(d)))
    return d.value


def synchronize() -> None:
    check(lib.kvc_device_synchronize())


def get_status(device: int | None = None, clear: bool = False) -> int:
    """Sticky kernel status bits (STATUS_*) of a device; synchronises it."""
    flags = ctypes.c_uint32(0)
    dev = current_device() if device is None else device
    check(lib.kvc_get_status(int(dev), ctypes.byref(flags), 1 if clear else 0))
    return flags.value
