"""The expert node's InferRequest / InferResponse bodies, restated -- TEST INFRASTRUCTURE ONLY.

Reference: ``common/infer_codec.cc:7-76`` (C++, the node) and ``common/protocol.py:503-577``
(Python, the coordinator), both over little-endian fixed fields:

    request   i32 expert_id, i32 batch_size, i32 hidden_dim, u32 input_dtype,
              u32 output_dtype, u32 n, then n activation bytes
    response  i32 status_code, i32 batch_size, i32 hidden_dim, u32 output_dtype, u32 n,
              then n output bytes

A body decodes only if every field and the whole payload are present and nothing trails
(``DecodeInferRequestBody`` returns false, ``decode_infer_request`` raises).  Pinned against
bodies made by both reference codecs (``tests/golden/infer_codec_golden.npz``).
"""
from __future__ import annotations

import struct

REQUEST_FIXED = struct.Struct("<iiiIII")
RESPONSE_FIXED = struct.Struct("<iiiII")


def encode(kind: str, fields, payload: bytes) -> bytes:
    st = REQUEST_FIXED if kind == "request" else RESPONSE_FIXED
    return st.pack(*[int(f) for f in fields], len(payload)) + bytes(payload)


def decode(kind: str, body: bytes):
    """(fields, payload), or None for a body the reference rejects."""
    st = REQUEST_FIXED if kind == "request" else RESPONSE_FIXED
    if len(body) < st.size:
        return None
    *fields, n = st.unpack_from(body, 0)
    if st.size + n != len(body):
        return None
    return tuple(fields), bytes(body[st.size:])
