"""fp16 / bf16 <-> fp32 bit codecs (CPU oracle; test infrastructure only).

Restates ``expert_node_v2/backend/activation_codec_v2.h``:

* ``DecodeFp16ToFloatV2`` (``:8-40``) and ``DecodeBf16ToFloatV2`` (``:42-47``): exact.
* ``EncodeFloatToFp16V2`` (``:49-81``): round-half-up on the dropped 13 bits
  (``mant + 0x1000``), flush below 2^-24, +-inf at overflow.
* ``EncodeFloatToBf16V2`` (``:83-88``): ``(bits + 0x8000) >> 16`` (round-half-up,
  not round-to-nearest-even; NaN payloads are not preserved).
"""
from __future__ import annotations

import numpy as np


def decode_bf16(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def encode_bf16_ref(x: np.ndarray) -> np.ndarray:
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x8000) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def encode_bf16_rne(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 (what torch ``.to(bfloat16)`` and ``__float2bfloat16`` do)."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    out = ((b + 0x7FFF + lsb) & 0xFFFFFFFF) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = np.where(nan, 0x7FC0, out)
    return out.astype(np.uint16)


def decode_fp16(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def encode_fp16_ref(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    mant = bits & 0x7FFFFF
    out = np.zeros(x.shape, dtype=np.int64)
    # subnormal / underflow branch (exp <= 0)
    sub = exp <= 0
    shift = np.clip(1 - exp, 0, 63)
    sub_m = (mant | 0x800000) >> shift
    sub_val = np.where(exp < -10, sign, sign | ((sub_m + 0x1000) >> 13))
    # overflow branch
    ovf = exp >= 31
    # normal branch
    half_mant = (mant + 0x1000) >> 13
    carry = half_mant == 0x400
    exp_n = np.where(carry, exp + 1, exp)
    half_mant = np.where(carry, 0, half_mant)
    norm_val = np.where(exp_n >= 31, sign | 0x7C00, sign | (exp_n << 10) | half_mant)
    out = np.where(sub, sub_val, np.where(ovf, sign | 0x7C00, norm_val))
    return out.astype(np.uint16)
