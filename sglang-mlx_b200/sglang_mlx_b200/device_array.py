"""DeviceArray: a minimal strided CUDA array owned by this package.

It plays the role `mx.array` plays for the reference (sglang_mlx/metal_kernels.py
passes mx.array objects straight to the extension): device memory comes from
libkvcache's allocator, the descriptor is handed to the C ABI without a DLPack
capsule round trip, and `__dlpack__` / `from_dlpack` exchange buffers with any
other DLPack framework.
"""

from __future__ import annotations

import ctypes
import math
import weakref

import numpy as np

from . import _lib, dlpack, dtypes

_lib_ref = _lib.lib


class _Buffer:
    """Owns one device allocation; freed when the last view is gone."""

    __slots__ = ("ptr", "nbytes", "device", "__weakref__")

    def __init__(self, nbytes: int, device: int):
        self.device = device
        self.nbytes = nbytes
        p = ctypes.c_void_p()
        prev = _lib.current_device()
        if prev != device:
            _lib.set_device(device)
        try:
            _lib.check(_lib_ref.kvc_malloc(ctypes.byref(p), ctypes.c_size_t(max(nbytes, 1))))
        finally:
            if prev != device:
                _lib.set_device(prev)
        self.ptr = p.value or 0
        weakref.finalize(self, _free, self.ptr)


def _free(ptr: int) -> None:
    try:
        _lib_ref.kvc_free(ctypes.c_void_p(ptr))
    except Exception:  # interpreter shutdown
        pass


class HostBuffer:
    """Pinned (page-locked) host memory exposed as a NumPy array."""

    def __init__(self, shape, dtype="float32"):
        self.dtype = dtypes.canonical(dtype)
        self.shape = tuple(int(s) for s in shape)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * dtypes.itemsize(self.dtype)
        p = ctypes.c_void_p()
        _lib.check(_lib_ref.kvc_malloc_host(ctypes.byref(p), ctypes.c_size_t(max(self.nbytes, 1))))
        self.ptr = p.value
        raw = (ctypes.c_uint8 * max(self.nbytes, 1)).from_address(self.ptr)
        self.array = np.frombuffer(raw, dtype=np.uint8, count=self.nbytes).view(
            dtypes.storage_dtype(self.dtype)).reshape(self.shape)
        weakref.finalize(self, _lib_ref.kvc_free_host, ctypes.c_void_p(self.ptr))

    def _dltensor(self):
        """(DLTensor, keepalive) describing this buffer as pinned host memory (kDLCUDAHost)."""
        from .dlpack import KDL_CUDA_HOST, make_dltensor

        return make_dltensor(self.ptr, self.shape, _contiguous_strides(self.shape), self.dtype, 0, KDL_CUDA_HOST)


def _contiguous_strides(shape) -> tuple:
    acc, st = 1, []
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    return tuple(reversed(st))


class DeviceArray:
    """A strided view of device memory: (buffer, element offset, shape, strides, dtype)."""

    __slots__ = ("_buf", "_offset", "shape", "strides", "dtype", "device", "_dl", "_dl_keep", "_foreign")

    def __init__(self, shape, dtype=dtypes.float32, device: int | None = None, *, _buf=None, _offset=0,
                 strides=None, _foreign=None):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtypes.canonical(dtype)
        self.strides = tuple(strides) if strides is not None else _contiguous_strides(self.shape)
        if _buf is None:
            dev = _lib.current_device() if device is None else int(device)
            _buf = _Buffer(self.nbytes_dense, dev)
        self._buf = _buf
        self._offset = int(_offset)
        self.device = _buf.device
        self._dl = None
        self._dl_keep = None
        self._foreign = _foreign

    # ---- construction ------------------------------------------------------
    @classmethod
    def empty(cls, shape, dtype=dtypes.float32, device: int | None = None) -> "DeviceArray":
        return cls(shape, dtype, device)

    @classmethod
    def zeros(cls, shape, dtype=dtypes.float32, device: int | None = None, stream=None) -> "DeviceArray":
        a = cls(shape, dtype, device)
        _lib.check(_lib_ref.kvc_memset_async(ctypes.c_void_p(a.ptr), 0, ctypes.c_size_t(a.nbytes_dense),
                                             _stream(stream)))
        return a

    @classmethod
    def from_numpy(cls, arr, dtype=None, device: int | None = None, stream=None) -> "DeviceArray":
        """Uploads `arr`.  With dtype='bfloat16' a float array is rounded to
        nearest even; a uint16 array is taken as raw bf16 bits."""
        arr = np.asarray(arr)
        name = dtypes.canonical(dtype if dtype is not None else arr.dtype)
        if name == dtypes.bfloat16:
            host = arr.astype(np.uint16) if arr.dtype == np.uint16 else dtypes.f32_to_bf16_bits(arr)
        else:
            host = arr.astype(dtypes.storage_dtype(name), copy=False)
        host = np.ascontiguousarray(host)
        a = cls(host.shape, name, device)
        if host.nbytes:
            _lib.check(_lib_ref.kvc_memcpy_async(ctypes.c_void_p(a.ptr), host.ctypes.data_as(ctypes.c_void_p),
                                                 ctypes.c_size_t(host.nbytes), 1, _stream(stream)))
            _lib.check(_lib_ref.kvc_stream_synchronize(_stream(stream)))
        return a

    @classmethod
    def from_dlpack(cls, obj) -> "DeviceArray":
        """Zero-copy view of another framework's CUDA array (keeps it alive)."""
        shape, strides, dt, dev_type, dev_id = dlpack.describe(obj)
        if dev_type not in (dlpack.KDL_CUDA, dlpack.KDL_CUDA_MANAGED):
            raise ValueError("from_dlpack: array is not on a CUDA device")
        ptr, keep = dlpack.as_dltensor(obj)
        data = (ptr.contents.data or 0) + ptr.contents.byte_offset

        class _Borrowed:
            __slots__ = ("ptr", "nbytes", "device", "__weakref__")

        b = _Borrowed()
        b.ptr, b.nbytes, b.device = data, 0, dev_id
        return cls(shape, dt, _buf=b, _offset=0, strides=strides, _foreign=(obj, keep))

    # ---- properties ---------------------------------------------------------
    @property
    def itemsize(self) -> int:
        return dtypes.itemsize(self.dtype)

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def size(self) -> int:
        return int(math.prod(self.shape))

    @property
    def nbytes_dense(self) -> int:
        return self.size * self.itemsize

    @property
    def nbytes(self) -> int:
        return self.nbytes_dense

    @property
    def ptr(self) -> int:
        return self._buf.ptr + self._offset * self.itemsize

    def is_contiguous(self) -> bool:
        return all(sh == 1 or st == ex for sh, st, ex in zip(self.shape, self.strides, _contiguous_strides(self.shape)))

    def __repr__(self) -> str:
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype}, device=cuda:{self.device})"

    def __len__(self) -> int:
        return self.shape[0]

    # ---- views --------------------------------------------------------------
    def _view(self, shape, strides, offset) -> "DeviceArray":
        return DeviceArray(shape, self.dtype, _buf=self._buf, _offset=offset, strides=strides, _foreign=self._foreign)

    def __getitem__(self, idx) -> "DeviceArray":
        if not isinstance(idx, tuple):
            idx = (idx,)
        if any(i is Ellipsis for i in idx):
            k = idx.index(Ellipsis)
            fill = self.ndim - (len(idx) - 1)
            idx = idx[:k] + (slice(None),) * fill + idx[k + 1:]
        if len(idx) > self.ndim:
            raise IndexError("too many indices")
        shape, strides, off = [], [], self._offset
        for d, (n, st) in enumerate(zip(self.shape, self.strides)):
            if d >= len(idx):
                shape.append(n)
                strides.append(st)
                continue
            i = idx[d]
            if isinstance(i, (int, np.integer)):
                i = int(i)
                if i < 0:
                    i += n
                if not 0 <= i < n:
                    raise IndexError(f"index {idx[d]} out of range for dim {d} of size {n}")
                off += i * st
            elif isinstance(i, slice):
                start, stop, step = i.indices(n)
                if step <= 0:
                    raise IndexError("only positive slice steps are supported")
                cnt = max(0, (stop - start + step - 1) // step)
                off += start * st
                shape.append(cnt)
                strides.append(st * step)
            else:
                raise TypeError("DeviceArray supports integer and slice indexing only")
        return self._view(tuple(shape), tuple(strides), off)

    def transpose(self, *axes) -> "DeviceArray":
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        if not axes:
            axes = tuple(reversed(range(self.ndim)))
        return self._view(tuple(self.shape[a] for a in axes), tuple(self.strides[a] for a in axes), self._offset)

    def reshape(self, *shape) -> "DeviceArray":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = list(shape)
        if -1 in shape:
            k = shape.index(-1)
            rest = int(math.prod(s for s in shape if s != -1))
            shape[k] = self.size // max(rest, 1)
        if int(math.prod(shape)) != self.size:
            raise ValueError(f"cannot reshape {self.shape} into {tuple(shape)}")
        if not self.is_contiguous():
            raise ValueError("reshape of a non-contiguous DeviceArray")
        return self._view(tuple(shape), _contiguous_strides(shape), self._offset)

    def expand_dims(self, axis: int) -> "DeviceArray":
        shape, strides = list(self.shape), list(self.strides)
        if axis < 0:
            axis += self.ndim + 1
        shape.insert(axis, 1)
        strides.insert(axis, strides[axis] * shape[axis + 1] if axis < len(strides) else 1)
        return self._view(tuple(shape), tuple(strides), self._offset)

    # ---- host transfer ---------------------------------------------------------
    def _span(self) -> tuple[int, int]:
        """(first element offset, element count) covered by the view."""
        if self.size == 0:
            return self._offset, 0
        lo = self._offset + sum((n - 1) * s for n, s in zip(self.shape, self.strides) if s < 0)
        hi = self._offset + sum((n - 1) * s for n, s in zip(self.shape, self.strides) if s > 0)
        return lo, hi - lo + 1

    def to_numpy(self, stream=None, raw: bool = False) -> np.ndarray:
        """Copies to the host.  bf16 comes back as float32 unless raw=True."""
        store = dtypes.storage_dtype(self.dtype)
        lo, count = self._span()
        host = np.empty(count, dtype=store)
        if count:
            src = self._buf.ptr + lo * self.itemsize
            _lib.check(_lib_ref.kvc_memcpy_async(host.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(src),
                                                 ctypes.c_size_t(count * self.itemsize), 2, _stream(stream)))
            _lib.check(_lib_ref.kvc_stream_synchronize(_stream(stream)))
        base = self._offset - lo
        out = np.lib.stride_tricks.as_strided(
            host[base:] if count else host, shape=self.shape,
            strides=tuple(s * self.itemsize for s in self.strides)).copy()
        if self.dtype == dtypes.bfloat16 and not raw:
            return dtypes.bf16_bits_to_f32(out).reshape(self.shape)
        return out

    numpy = to_numpy

    def __array__(self, dtype=None, copy=None):
        a = self.to_numpy()
        return a.astype(dtype) if dtype is not None else a

    def copy_from_host(self, host, stream=None) -> None:
        """Async upload of a contiguous host array of the same byte size (pinned for overlap)."""
        h = host.array if isinstance(host, HostBuffer) else np.ascontiguousarray(host)
        if not self.is_contiguous() or h.nbytes != self.nbytes_dense:
            raise ValueError("copy_from_host needs a contiguous destination of the same byte size")
        _lib.check(_lib_ref.kvc_memcpy_async(ctypes.c_void_p(self.ptr), h.ctypes.data_as(ctypes.c_void_p),
                                             ctypes.c_size_t(h.nbytes), 1, _stream(stream)))

    def copy_to_host(self, host, stream=None) -> None:
        """Async download into a contiguous host array of the same byte size."""
        h = host.array if isinstance(host, HostBuffer) else host
        if not self.is_contiguous() or h.nbytes != self.nbytes_dense or not h.flags.c_contiguous:
            raise ValueError("copy_to_host needs contiguous arrays of the same byte size")
        _lib.check(_lib_ref.kvc_memcpy_async(h.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(self.ptr),
                                             ctypes.c_size_t(h.nbytes), 2, _stream(stream)))

    def fill_zero(self, stream=None) -> None:
        if not self.is_contiguous():
            raise ValueError("fill_zero needs a contiguous array")
        _lib.check(_lib_ref.kvc_memset_async(ctypes.c_void_p(self.ptr), 0, ctypes.c_size_t(self.nbytes_dense),
                                             _stream(stream)))

    # ---- DLPack ---------------------------------------------------------------
    def _dltensor(self) -> dlpack.DLTensor:
        if self._dl is None:
            self._dl, self._dl_keep = dlpack.make_dltensor(self.ptr, self.shape, self.strides, self.dtype, self.device)
        return self._dl

    def __dlpack_device__(self):
        return (dlpack.KDL_CUDA, self.device)

    def __dlpack__(self, stream=None, max_version=None, dl_device=None, copy=None):
        # Work is issued on the legacy default stream or on streams the caller
        # synchronises; nothing to order here.
        return _export_capsule(self)


# Exported DLManagedTensors stay referenced here until the consumer calls the deleter.
_EXPORTED: dict[int, tuple] = {}


@dlpack._DELETER
def _exported_deleter(mt_ptr):
    _EXPORTED.pop(ctypes.cast(mt_ptr, ctypes.c_void_p).value, None)


def _export_capsule(arr: DeviceArray):
    mt = dlpack.DLManagedTensor()
    t, keep = dlpack.make_dltensor(arr.ptr, arr.shape, arr.strides, arr.dtype, arr.device)
    mt.dl_tensor = t
    mt.manager_ctx = None
    mt.deleter = _exported_deleter
    addr = ctypes.addressof(mt)
    _EXPORTED[addr] = (mt, keep, arr)
    return dlpack._pyapi.PyCapsule_New(ctypes.c_void_p(addr), b"dltensor", None)


def _stream(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(getattr(stream, "handle", stream))


def asarray(obj, dtype=None, device: int | None = None) -> DeviceArray:
    """DeviceArray view of a DLPack device array, or an upload of host data."""
    if isinstance(obj, DeviceArray):
        return obj
    if hasattr(obj, "__dlpack_device__"):
        dev_type, _ = obj.__dlpack_device__()
        if dev_type in (dlpack.KDL_CUDA, dlpack.KDL_CUDA_MANAGED):
            return DeviceArray.from_dlpack(obj)
    return DeviceArray.from_numpy(np.asarray(obj), dtype=dtype, device=device)


class Stream:
    """An owned CUDA stream (non-blocking)."""

    def __init__(self):
        p = ctypes.c_void_p()
        _lib.check(_lib_ref.kvc_stream_create(ctypes.byref(p)))
        self.handle = p.value
        weakref.finalize(self, _lib_ref.kvc_stream_destroy, ctypes.c_void_p(self.handle))

    def synchronize(self) -> None:
        _lib.check(_lib_ref.kvc_stream_synchronize(ctypes.c_void_p(self.handle)))

    def wait(self, event: "Event") -> None:
        """Work queued on this stream from now on waits for `event`."""
        _lib.check(_lib_ref.kvc_stream_wait_event(ctypes.c_void_p(self.handle), ctypes.c_void_p(event.handle)))


class Graph:
    """A captured sequence of libkvcache work, replayed with one launch.

        g = Graph.capture(stream, fn)   # runs fn() under stream capture
        g.replay(stream)

    Every call inside `fn` must pass `stream=stream`; arrays it touches must be
    allocated beforehand and stay alive as long as the graph."""

    def __init__(self, handle: int):
        self.handle = handle
        weakref.finalize(self, _lib_ref.kvc_graph_destroy, ctypes.c_void_p(handle))

    @classmethod
    def capture(cls, stream: "Stream", fn) -> "Graph":
        _lib.check(_lib_ref.kvc_stream_begin_capture(ctypes.c_void_p(stream.handle)))
        try:
            fn()
        finally:
            h = ctypes.c_void_p()
            rc = _lib_ref.kvc_stream_end_capture(ctypes.c_void_p(stream.handle), ctypes.byref(h))
        _lib.check(rc)
        return cls(h.value)

    def replay(self, stream: "Stream") -> None:
        _lib.check(_lib_ref.kvc_graph_launch(ctypes.c_void_p(self.handle), ctypes.c_void_p(stream.handle)))


class Event:
    """A CUDA event for device-side timing."""

    def __init__(self):
        p = ctypes.c_void_p()
        _lib.check(_lib_ref.kvc_event_create(ctypes.byref(p)))
        self.handle = p.value
        weakref.finalize(self, _lib_ref.kvc_event_destroy, ctypes.c_void_p(self.handle))

    def record(self, stream=None) -> None:
        _lib.check(_lib_ref.kvc_event_record(ctypes.c_void_p(self.handle), _stream(stream)))

    def synchronize(self) -> None:
        _lib.check(_lib_ref.kvc_event_synchronize(ctypes.c_void_p(self.handle)))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0.0)
        _lib.check(_lib_ref.kvc_event_elapsed_ms(ctypes.c_void_p(self.handle), ctypes.c_void_p(end.handle),
                                                 ctypes.byref(ms)))
        return float(ms.value)
