"""Build and load the compiled CPU checkers in ``oracle/_ref/`` (test infrastructure only).

* ``libexpert_oracle.so``: ``oracle/expert_ref.c``, our plain-C restatement of the
  reference's scalar expert.  Always buildable (gcc only).
* ``libref_expert.so``: the reference's own C++ expert code, compiled from its
  unmodified sources by ``oracle/Makefile`` when the reference tree is present
  (``CONSTELLATION_REFERENCE_ROOT``); on a machine without it the prebuilt file
  that travelled with the repository is used as is.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
ORACLE_SO = OUT / "libexpert_oracle.so"
REF_SO = OUT / "libref_expert.so"


def reference_root() -> Path | None:
    """The reference checkout: ``$CONSTELLATION_REFERENCE_ROOT``, else a ``reference``
    directory beside this repository; None when neither holds the reference sources."""
    default = HERE.parent.parent / "reference"
    root = Path(os.environ.get("CONSTELLATION_REFERENCE_ROOT", str(default)))
    marker = root / "expert_node_v2" / "backend" / "expert_reference_v2.cc"
    return root if marker.is_file() else None


def build(verbose: bool = False) -> None:
    """Build both libraries (the reference one only when its sources are present)."""
    out = None if verbose else subprocess.DEVNULL
    subprocess.run(["make", "-C", str(HERE), "all"], check=True, stdout=out)
    root = reference_root()
    if root is not None:
        subprocess.run(["make", "-C", str(HERE), f"REF={root}", "ref"], check=True, stdout=out)


_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctype)


_oracle_lib = None
_ref_lib = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle_lib
    if _oracle_lib is None:
        if not ORACLE_SO.is_file():
            build()
        lib = ctypes.CDLL(str(ORACLE_SO))
        lib.oracle_expert_lut.restype = ctypes.c_int
        lib.oracle_expert_lut.argtypes = [_u8p, _f32p, _u8p, _f32p, _u8p, _f32p] + [ctypes.c_int] * 4 + \
            [_f32p, ctypes.c_int, _f32p, _f32p]
        lib.oracle_decode_e4m3fn_ref.restype = ctypes.c_float
        lib.oracle_decode_e4m3fn_ref.argtypes = [ctypes.c_int]
        _oracle_lib = lib
    return _oracle_lib


def ref_available() -> bool:
    return REF_SO.is_file()


def ref_lib() -> ctypes.CDLL:
    global _ref_lib
    if _ref_lib is None:
        if not REF_SO.is_file():
            raise FileNotFoundError(f"{REF_SO} is not built (the reference sources were absent)")
        lib = ctypes.CDLL(str(REF_SO))
        lib.ref_fill_dummy.restype = ctypes.c_int
        lib.ref_fill_dummy.argtypes = [ctypes.c_int] * 4 + [_u8p, _f32p, _u8p, _f32p, _u8p, _f32p]
        lib.ref_dummy_input.restype = None
        lib.ref_dummy_input.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, _u16p]
        wargs = [_u8p, _f32p, _u8p, _f32p, _u8p, _f32p] + [ctypes.c_int] * 4
        lib.ref_expert_reference.restype = ctypes.c_int
        lib.ref_expert_reference.argtypes = wargs + [_u16p, ctypes.c_int, ctypes.c_int, _u16p, _f32p]
        lib.ref_expert_cpu.restype = ctypes.c_int
        lib.ref_expert_cpu.argtypes = wargs + [_u16p, ctypes.c_int, _u16p, ctypes.c_int, _f32p,
                                               ctypes.c_int]
        lib.ref_decode_fp8.restype = ctypes.c_float
        lib.ref_decode_fp8.argtypes = [ctypes.c_int, ctypes.c_int]
        lib.ref_encode_bf16.restype = ctypes.c_uint16
        lib.ref_encode_bf16.argtypes = [ctypes.c_float]
        lib.ref_encode_fp16.restype = ctypes.c_uint16
        lib.ref_encode_fp16.argtypes = [ctypes.c_float]
        lib.ref_decode_bf16.restype = ctypes.c_float
        lib.ref_decode_bf16.argtypes = [ctypes.c_uint16]
        lib.ref_decode_fp16.restype = ctypes.c_float
        lib.ref_decode_fp16.argtypes = [ctypes.c_uint16]
        LL, LLP, VP = ctypes.c_longlong, ctypes.POINTER(ctypes.c_longlong), ctypes.c_void_p
        I32, U32 = ctypes.c_int32, ctypes.c_uint32
        lib.ref_encode_infer_request.restype = LL
        lib.ref_encode_infer_request.argtypes = [I32, I32, I32, U32, U32, VP, LL, VP, LL]
        lib.ref_encode_infer_response.restype = LL
        lib.ref_encode_infer_response.argtypes = [I32, I32, I32, U32, VP, LL, VP, LL]
        for name in ("ref_decode_infer_request", "ref_decode_infer_response"):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [VP, LL, LLP, VP, LL, LLP]
        _ref_lib = lib
    return _ref_lib


class ExpertBytes:
    """The six tensors of one expert in the reference layout (``expert_format_v2.h:59-86``)."""

    def __init__(self, w_up, s_up, w_gate, s_gate, w_down, s_down, block: int = 128):
        c = np.ascontiguousarray
        self.w_up = c(w_up, dtype=np.uint8)
        self.s_up = c(s_up, dtype=np.float32)
        self.w_gate = c(w_gate, dtype=np.uint8)
        self.s_gate = c(s_gate, dtype=np.float32)
        self.w_down = c(w_down, dtype=np.uint8)
        self.s_down = c(s_down, dtype=np.float32)
        self.block = block

    @property
    def inter(self) -> int:
        return int(self.w_up.shape[0])

    @property
    def hidden(self) -> int:
        return int(self.w_up.shape[1])

    def ptrs(self):
        return (_ptr(self.w_up, _u8p), _ptr(self.s_up, _f32p), _ptr(self.w_gate, _u8p),
                _ptr(self.s_gate, _f32p), _ptr(self.w_down, _u8p), _ptr(self.s_down, _f32p))


def dummy_expert(hidden: int, inter: int, block: int = 128) -> ExpertBytes:
    """The reference's deterministic dummy bundle (``dummy_expert_data_v2.cc:9-132``)."""
    br, bc = (inter + block - 1) // block, (hidden + block - 1) // block
    wu = np.empty((inter, hidden), np.uint8)
    wg = np.empty((inter, hidden), np.uint8)
    wd = np.empty((hidden, inter), np.uint8)
    su = np.empty((br, bc), np.float32)
    sg = np.empty((br, bc), np.float32)
    sd = np.empty((bc, br), np.float32)
    e = ExpertBytes(wu, su, wg, sg, wd, sd, block)
    rc = ref_lib().ref_fill_dummy(hidden, inter, block, block, *e.ptrs())
    if rc != 0:
        raise RuntimeError("FillDummyExpertBundleV2 produced an invalid bundle")
    return e


def dummy_expert_formula(hidden: int, inter: int, block: int = 128) -> ExpertBytes:
    """Same bundle as ``dummy_expert`` computed in numpy (usable without the reference)."""
    i = np.arange(inter * hidden, dtype=np.int64)
    wu = ((i * 7 + 3) & 0xFF).astype(np.uint8).reshape(inter, hidden)
    wg = ((i * 11 + 5) & 0xFF).astype(np.uint8).reshape(inter, hidden)
    wd = ((i * 13 + 17) & 0xFF).astype(np.uint8).reshape(hidden, inter)
    br, bc = (inter + block - 1) // block, (hidden + block - 1) // block
    rb = np.arange(br, dtype=np.float32)[:, None]
    cb = np.arange(bc, dtype=np.float32)[None, :]
    su = (np.float32(0.010) + np.float32(0.0005) * rb + np.float32(0.00005) * cb).astype(np.float32)
    sg = (np.float32(0.020) + np.float32(0.0003) * rb + np.float32(0.00007) * cb).astype(np.float32)
    rb2 = np.arange(bc, dtype=np.float32)[:, None]
    cb2 = np.arange(br, dtype=np.float32)[None, :]
    sd = (np.float32(0.005) + np.float32(0.001) * rb2 + np.float32(0.0001) * cb2).astype(np.float32)
    return ExpertBytes(wu, su, wg, sg, wd, sd, block)


def dummy_input_formula(hidden: int) -> np.ndarray:
    """``x[i] = sin(0.0005 i)`` in float32 (``dummy_expert_data_v2.cc:134-150``)."""
    return np.sin(np.float32(0.0005) * np.arange(hidden, dtype=np.float32)).astype(np.float32)


def oracle_expert_lut(e: ExpertBytes, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Our C restatement: ``x [n, H] fp32`` -> (``h [n, I]``, ``y [n, H]``) fp32."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    n = x.shape[0]
    h = np.empty((n, e.inter), np.float32)
    y = np.empty((n, e.hidden), np.float32)
    rc = oracle_lib().oracle_expert_lut(*e.ptrs(), e.inter, e.hidden, e.block, e.block,
                                        _ptr(x, _f32p), n, _ptr(h, _f32p), _ptr(y, _f32p))
    if rc != 0:
        raise RuntimeError(f"oracle_expert_lut failed rc={rc}")
    return h, y


def ref_expert_reference(e: ExpertBytes, x_bits: np.ndarray, in_dtype: int, out_dtype: int):
    """Reference ``RunExpertReferenceV2`` per row of ``x_bits [n, H] uint16`` -> (y bits, h)."""
    x_bits = np.ascontiguousarray(np.atleast_2d(x_bits), dtype=np.uint16)
    n = x_bits.shape[0]
    y = np.empty((n, e.hidden), np.uint16)
    h = np.empty((n, e.inter), np.float32)
    lib = ref_lib()
    for t in range(n):
        rc = lib.ref_expert_reference(*e.ptrs(), e.inter, e.hidden, e.block, e.block,
                                      _ptr(x_bits[t], _u16p), in_dtype, out_dtype,
                                      _ptr(y[t], _u16p), _ptr(h[t], _f32p))
        if rc != 0:
            raise RuntimeError(f"RunExpertReferenceV2 failed rc={rc}")
    return y, h


def ref_expert_cpu(e: ExpertBytes, x_bits: np.ndarray, in_dtype: int, out_dtype: int,
                   threads: int) -> np.ndarray:
    """Reference OpenMP CPU backend, one batch-1 call per row (the timed CPU baseline)."""
    x_bits = np.ascontiguousarray(np.atleast_2d(x_bits), dtype=np.uint16)
    n = x_bits.shape[0]
    y = np.empty((n, e.hidden), np.uint16)
    scratch = np.empty(e.inter, np.float32)
    lib = ref_lib()
    for t in range(n):
        rc = lib.ref_expert_cpu(*e.ptrs(), e.inter, e.hidden, e.block, e.block,
                                _ptr(x_bits[t], _u16p), in_dtype, _ptr(y[t], _u16p), out_dtype,
                                _ptr(scratch, _f32p), threads)
        if rc != 0:
            raise RuntimeError(f"RunExpertCpuV2 kernels failed rc={rc}")
    return y


def _buf(data: bytes):
    return (ctypes.c_uint8 * max(1, len(data))).from_buffer_copy(data or b"\0")


def ref_encode_infer(kind: str, fields, payload: bytes) -> bytes:
    """The reference C++ ``Encode{InferRequest,InferResponse}Body`` (common/infer_codec.cc)."""
    lib = ref_lib()
    out = (ctypes.c_uint8 * (len(payload) + 64))()
    src = _buf(payload)
    fn = lib.ref_encode_infer_request if kind == "request" else lib.ref_encode_infer_response
    n = fn(*[int(f) for f in fields], ctypes.addressof(src), len(payload), ctypes.addressof(out), len(out))
    if n < 0:
        raise RuntimeError("reference encoder: buffer too small")
    return bytes(out[:n])


def ref_decode_infer(kind: str, body: bytes):
    """The reference C++ ``Decode*Body``: (fields, payload), or None when it rejects the body."""
    lib = ref_lib()
    src = _buf(body)
    fields = (ctypes.c_longlong * 5)()
    payload = (ctypes.c_uint8 * max(1, len(body)))()
    n = ctypes.c_longlong(0)
    fn = lib.ref_decode_infer_request if kind == "request" else lib.ref_decode_infer_response
    if not fn(ctypes.addressof(src), len(body), fields, ctypes.addressof(payload), len(payload), ctypes.byref(n)):
        return None
    k = 5 if kind == "request" else 4
    return tuple(int(f) for f in fields[:k]), bytes(payload[:n.value])
