"""The expert node's InferRequest / InferResponse bodies, through the library's codec.

Same names, dict keys and errors as the reference coordinator's codec
(``common/protocol.py:503-577``): ``encode_*`` take a dict and return ``bytes`` (``ValueError``
for a payload that is not bytes-like or a field outside its i32 / u32 range); ``decode_*``
return a dict and raise ``ProtocolError`` for a body that ends inside a field or the
payload, or has trailing bytes.  The bytes are written and read by
``cst_encode_infer_request`` & co. -- host code of ``libconstellation_b200.so``, the same
routines ``cst_serve_infer_request`` runs on the node side -- so coordinator and node share
one implementation of the wire format (``common/infer_codec.cc:7-76`` in the reference).
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import CstInferRequest, CstInferResponse


class ProtocolError(RuntimeError):
    pass


def _i32(x) -> int:
    x = int(x)
    if x < -0x80000000 or x > 0x7FFFFFFF:
        raise ValueError(f"i32 out of range: {x}")
    return x


def _u32(x) -> int:
    x = int(x)
    if x < 0 or x > 0xFFFFFFFF:
        raise ValueError(f"u32 out of range: {x}")
    return x


def _bytes_arg(data, name: str):
    if not isinstance(data, (bytes, bytearray)):
        raise ValueError(f"{name} must be bytes-like")
    n = len(data)
    buf = (ctypes.c_uint8 * max(n, 1)).from_buffer_copy(bytes(data) if n else b"\0")
    return buf, n


def _encode(fn, msg_struct) -> bytes:
    need = ctypes.c_int64(0)
    fn(ctypes.byref(msg_struct), None, 0, ctypes.byref(need))  # size query
    out = (ctypes.c_uint8 * max(int(need.value), 1))()
    _lib.check(fn(ctypes.byref(msg_struct), ctypes.addressof(out), len(out), ctypes.byref(need)))
    return ctypes.string_at(ctypes.addressof(out), need.value)


def encode_infer_request(msg) -> bytes:
    buf, n = _bytes_arg(msg["activation"], "activation")
    m = CstInferRequest(_i32(msg["expert_id"]), _i32(msg["batch_size"]), _i32(msg["hidden_dim"]),
                        _u32(msg["input_dtype"]), _u32(msg["output_dtype"]), _u32(n), ctypes.addressof(buf))
    return _encode(_lib.lib.cst_encode_infer_request, m)


def encode_infer_response(msg) -> bytes:
    buf, n = _bytes_arg(msg["output"], "output")
    m = CstInferResponse(_i32(msg["status_code"]), _i32(msg["batch_size"]), _i32(msg["hidden_dim"]),
                         _u32(msg["output_dtype"]), _u32(n), ctypes.addressof(buf))
    return _encode(_lib.lib.cst_encode_infer_response, m)


def _decode(fn, body, m):
    body = bytes(body)
    buf = (ctypes.c_uint8 * max(len(body), 1)).from_buffer_copy(body or b"\0")
    rc = fn(ctypes.addressof(buf), len(body), ctypes.byref(m))
    if rc != _lib.CST_OK:
        raise ProtocolError(_lib.last_error())
    return body


def decode_infer_request(body: bytes) -> dict:
    m = CstInferRequest()
    body = _decode(_lib.lib.cst_decode_infer_request, body, m)
    n = int(m.activation_bytes)
    return {
        "expert_id": m.expert_id,
        "batch_size": m.batch_size,
        "hidden_dim": m.hidden_dim,
        "input_dtype": int(m.input_dtype),
        "output_dtype": int(m.output_dtype),
        "activation": body[len(body) - n:],
    }


def decode_infer_response(body: bytes) -> dict:
    m = CstInferResponse()
    body = _decode(_lib.lib.cst_decode_infer_response, body, m)
    n = int(m.output_bytes)
    return {
        "status_code": m.status_code,
        "batch_size": m.batch_size,
        "hidden_dim": m.hidden_dim,
        "output_dtype": int(m.output_dtype),
        "output": body[len(body) - n:],
    }
