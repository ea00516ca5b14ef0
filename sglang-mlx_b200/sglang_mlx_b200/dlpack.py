"""DLPack structs (restated from the public DLPack specification) and the
conversion of Python array objects into `DLTensor*` arguments for libkvcache.

Accepted inputs: this package's DeviceArray and HostBuffer (descriptors built
directly, no capsule), or any object implementing the DLPack protocol
(`__dlpack__`, e.g. a CUDA torch tensor, a CuPy array or a NumPy array).
"""

from __future__ import annotations

import ctypes

from . import dtypes

KDL_CPU = 1
KDL_CUDA = 2
KDL_CUDA_HOST = 3
KDL_CUDA_MANAGED = 13


class DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class DLTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("device", DLDevice),
        ("ndim", ctypes.c_int32),
        ("dtype", DLDataType),
        ("shape", ctypes.POINTER(ctypes.c_int64)),
        ("strides", ctypes.POINTER(ctypes.c_int64)),
        ("byte_offset", ctypes.c_uint64),
    ]


class DLManagedTensor(ctypes.Structure):
    pass


_DELETER = ctypes.CFUNCTYPE(None, ctypes.POINTER(DLManagedTensor))
DLManagedTensor._fields_ = [
    ("dl_tensor", DLTensor),
    ("manager_ctx", ctypes.c_void_p),
    ("deleter", _DELETER),
]

_pyapi = ctypes.pythonapi
_pyapi.PyCapsule_GetPointer.restype = ctypes.c_void_p
_pyapi.PyCapsule_GetPointer.argtypes = [ctypes.py_object, ctypes.c_char_p]
_pyapi.PyCapsule_New.restype = ctypes.py_object
_pyapi.PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
_pyapi.PyCapsule_IsValid.restype = ctypes.c_int
_pyapi.PyCapsule_IsValid.argtypes = [ctypes.py_object, ctypes.c_char_p]


def make_dltensor(ptr: int, shape, strides, dtype: str, device_id: int, device_type: int = KDL_CUDA):
    """Builds a DLTensor (and the arrays it points to) for a raw buffer.

    Returns (tensor, keepalive): keep `keepalive` referenced while the tensor
    is in use.
    """
    nd = len(shape)
    shp = (ctypes.c_int64 * max(nd, 1))(*shape)
    std = (ctypes.c_int64 * max(nd, 1))(*strides)
    code, bits = dtypes.dl_code_bits(dtype)
    t = DLTensor()
    t.data = ctypes.c_void_p(ptr)
    t.device = DLDevice(device_type, device_id)
    t.ndim = nd
    t.dtype = DLDataType(code, bits, 1)
    t.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
    t.strides = ctypes.cast(std, ctypes.POINTER(ctypes.c_int64))
    t.byte_offset = 0
    return t, (shp, std)


class _ForeignView:
    """A borrowed DLTensor read out of a producer's `__dlpack__` capsule."""

    __slots__ = ("capsule", "managed")

    def __init__(self, obj, stream=None):
        try:
            cap = obj.__dlpack__(stream=stream) if stream is not None else obj.__dlpack__()
        except TypeError:
            cap = obj.__dlpack__()
        if not _pyapi.PyCapsule_IsValid(cap, b"dltensor"):
            raise TypeError("object's __dlpack__ did not return a 'dltensor' capsule")
        addr = _pyapi.PyCapsule_GetPointer(cap, b"dltensor")
        self.capsule = cap  # the producer's capsule destructor frees it
        self.managed = DLManagedTensor.from_address(addr)

    @property
    def tensor(self) -> DLTensor:
        return self.managed.dl_tensor


def as_dltensor(obj, name: str = "tensor"):
    """Returns (ctypes pointer to a DLTensor, keepalive) for `obj`."""
    from .device_array import DeviceArray, HostBuffer

    if obj is None:
        return None, None
    if isinstance(obj, DeviceArray):
        t = obj._dltensor()
        return ctypes.pointer(t), obj
    if isinstance(obj, HostBuffer):
        t, keep = obj._dltensor()
        return ctypes.pointer(t), (obj, keep)
    if hasattr(obj, "__dlpack__"):
        view = _ForeignView(obj)
        return ctypes.pointer(view.managed.dl_tensor), view
    raise TypeError(f"{name}: expected a DeviceArray or a DLPack-capable device array, got {type(obj).__name__}")


def describe(obj) -> tuple[tuple, tuple, str, int, int]:
    """(shape, strides in elements, dtype name, device_type, device_id) of any accepted array."""
    ptr, keep = as_dltensor(obj)
    t = ptr.contents
    nd = t.ndim
    shape = tuple(t.shape[i] for i in range(nd))
    if t.strides:
        strides = tuple(t.strides[i] for i in range(nd))
    else:
        acc, st = 1, []
        for s in reversed(shape):
            st.append(acc)
            acc *= s
        strides = tuple(reversed(st))
    dt = dtypes.from_dl(t.dtype.code, t.dtype.bits)
    del keep
    return shape, strides, dt, t.device.device_type, t.device.device_id
