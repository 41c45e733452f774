"""A torch view of memory this library owns (DLPack over ctypes).

The peer-exchange buffers come from ``cst_ipc_alloc`` (``cudaMalloc`` + an IPC handle), not
from torch's allocator, but the layer entry points take torch tensors.  ``view`` builds a
DLPack capsule over a raw pointer and hands it to ``torch.utils.dlpack.from_dlpack``: the
tensor aliases the memory and does not own it -- the caller keeps the allocation alive (and
frees it) and must not use the view after that.
"""
from __future__ import annotations

import ctypes

import torch

_KDL_CPU, _KDL_CUDA = 1, 2
_KDL_INT, _KDL_UINT, _KDL_FLOAT, _KDL_BFLOAT = 0, 1, 2, 4
_CODES = {torch.float32: (_KDL_FLOAT, 32), torch.float16: (_KDL_FLOAT, 16), torch.bfloat16: (_KDL_BFLOAT, 16),
          torch.int32: (_KDL_INT, 32), torch.uint8: (_KDL_UINT, 8)}


class _DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class _DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class _DLTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("device", _DLDevice), ("ndim", ctypes.c_int32),
                ("dtype", _DLDataType), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("strides", ctypes.POINTER(ctypes.c_int64)), ("byte_offset", ctypes.c_uint64)]


_Deleter = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


class _DLManagedTensor(ctypes.Structure):
    _fields_ = [("dl_tensor", _DLTensor), ("manager_ctx", ctypes.c_void_p), ("deleter", _Deleter)]


_PyCapsule_New = ctypes.pythonapi.PyCapsule_New
_PyCapsule_New.restype = ctypes.py_object
_PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]

# every managed struct handed out stays referenced here: torch may call its deleter
# (a no-op) at any time until the view dies, and the view never owns the memory
_keep: dict[int, tuple] = {}


@_Deleter
def _release(p):
    _keep.pop(int(p or 0), None)


def view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Contiguous ``shape`` tensor of ``dtype`` over ``ptr`` on ``device`` (cuda or cpu)."""
    if dtype not in _CODES:
        raise TypeError(f"unsupported dtype {dtype}")
    device = torch.device(device)
    shape = tuple(int(s) for s in shape)
    dims = (ctypes.c_int64 * max(len(shape), 1))(*shape)
    code, bits = _CODES[dtype]
    mt = _DLManagedTensor()
    mt.dl_tensor.data = ptr
    if device.type == "cuda":
        idx = device.index if device.index is not None else torch.cuda.current_device()
        mt.dl_tensor.device = _DLDevice(_KDL_CUDA, idx)
    elif device.type == "cpu":
        mt.dl_tensor.device = _DLDevice(_KDL_CPU, 0)
    else:
        raise TypeError(f"unsupported device {device}")
    mt.dl_tensor.ndim = len(shape)
    mt.dl_tensor.dtype = _DLDataType(code, bits, 1)
    mt.dl_tensor.shape = ctypes.cast(dims, ctypes.POINTER(ctypes.c_int64))
    mt.dl_tensor.strides = None
    mt.dl_tensor.byte_offset = 0
    mt.manager_ctx = None
    mt.deleter = _release
    _keep[ctypes.addressof(mt)] = (mt, dims)
    capsule = _PyCapsule_New(ctypes.addressof(mt), b"dltensor", None)
    return torch.utils.dlpack.from_dlpack(capsule)
