"""FP8 E4M3 decode, block dequant and block quantizer (CPU oracle; test infrastructure only).

References restated here:

* ``expert_node_v2/backend/fp8_lut_v2.cc:47-66`` ``decode_torch_e4m3fn_byte``: the
  reference node's LUT for ``float8_e4m3fn``.  Bias 7, subnormals ``m/8 * 2^-6``,
  and the quirk that ``S.1111.111`` (0x7F / 0xFF) decodes to +-448 instead of NaN
  (``fp8_lut_v2.cc:59-61``).
* ``server/fp8_utils.py:4-39`` ``dequant_fp8_weight_blockwise``: ``out[r0:r1, c0:c1]
  = w.float() * scale_inv[bi, bj]`` over ``block_size`` x ``block_size`` blocks with
  ceil-div block counts (ragged last blocks allowed).  ``weight_fp8.float()`` is
  torch's true e4m3fn decode, where 0x7F / 0xFF are NaN.
* The synthetic quantizer of the benchmark configurations (config 0): per
  128x128 block ``s = amax / 448``, ``q = round_to_e4m3fn(W / s)`` saturating,
  ``s`` stored as ``scale_inv`` -- exactly what ``dequant_fp8_weight_blockwise``
  multiplies by.  The reference itself ships no quantizer (checkpoints arrive
  pre-quantized), so this one is defined by the benchmark configuration.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def _decode_e4m3_byte(v: int, *, ref_quirk: bool) -> float:
    sign = -1.0 if (v >> 7) & 1 else 1.0
    exp = (v >> 3) & 0xF
    mant = v & 0x7
    if exp == 0:
        return sign * (mant / 8.0) * 2.0 ** (1 - 7)
    if exp == 0xF and mant == 0x7:
        return sign * 448.0 if ref_quirk else float("nan")
    return sign * (1.0 + mant / 8.0) * 2.0 ** (exp - 7)


#: 256-entry LUT of the reference node (``fp8_lut_v2.cc:47-66``): 0x7F/0xFF -> +-448.
E4M3FN_REF_LUT = np.array([_decode_e4m3_byte(i, ref_quirk=True) for i in range(256)],
                          dtype=np.float32)
#: True ``float8_e4m3fn`` decode (what ``tensor.float()`` does): 0x7F/0xFF -> NaN.
E4M3FN_LUT = np.array([_decode_e4m3_byte(i, ref_quirk=False) for i in range(256)],
                      dtype=np.float32)


def decode_e4m3fn(b: np.ndarray, *, ref_quirk: bool = False) -> np.ndarray:
    """Decode uint8 E4M3FN bytes to float32 (``ref_quirk`` selects the node LUT)."""
    lut = E4M3FN_REF_LUT if ref_quirk else E4M3FN_LUT
    return lut[np.asarray(b, dtype=np.uint8)]


# Sorted finite non-negative E4M3FN magnitudes and their byte codes (0x00..0x7E).
_POS_CODES = np.arange(0x7F, dtype=np.uint8)
_POS_VALUES = E4M3FN_LUT[_POS_CODES].astype(np.float64)


def encode_e4m3fn_rne(v: np.ndarray) -> np.ndarray:
    """float32 -> E4M3FN bytes, round-to-nearest-even, saturating at +-448.

    NaN inputs map to 0x7F (the e4m3fn NaN code).  The grid search is exact:
    every finite e4m3fn value and every midpoint is representable in float64.
    """
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v.astype(np.float64))
    a_clip = np.minimum(a, E4M3_MAX)
    hi = np.searchsorted(_POS_VALUES, a_clip, side="left")  # first value >= a
    hi = np.clip(hi, 0, len(_POS_VALUES) - 1)
    lo = np.clip(hi - 1, 0, len(_POS_VALUES) - 1)
    v_hi = _POS_VALUES[hi]
    v_lo = _POS_VALUES[lo]
    d_hi = v_hi - a_clip
    d_lo = a_clip - v_lo
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((_POS_CODES[hi] & 1) == 0))
    pick_hi |= (hi == lo)
    code = np.where(pick_hi, _POS_CODES[hi], _POS_CODES[lo]).astype(np.uint8)
    code = np.where(v_hi == a_clip, _POS_CODES[hi], code).astype(np.uint8)
    neg = np.signbit(v)
    code = np.where(neg, code | np.uint8(0x80), code).astype(np.uint8)
    code = np.where(np.isnan(v), np.uint8(0x7F), code).astype(np.uint8)
    return code


def block_grid(rows: int, cols: int, block: int = 128) -> tuple[int, int]:
    return (rows + block - 1) // block, (cols + block - 1) // block


def expand_block_scale(scale_inv: np.ndarray, rows: int, cols: int, block: int = 128) -> np.ndarray:
    """Broadcast a ``[ceil(r/b), ceil(c/b)]`` scale grid to ``[rows, cols]`` (ragged crop)."""
    s = np.repeat(np.repeat(np.asarray(scale_inv, dtype=np.float32), block, axis=0), block, axis=1)
    return s[:rows, :cols]


def dequant_fp8_weight_blockwise(w_u8: np.ndarray, scale_inv: np.ndarray, block_size: int = 128,
                                 *, ref_quirk: bool = False) -> np.ndarray:
    """Restates ``server/fp8_utils.py:4-39`` (shape checks ``:9-25``, block loop ``:31-37``)."""
    w_u8 = np.asarray(w_u8, dtype=np.uint8)
    if w_u8.ndim != 2:
        raise RuntimeError(f"expected 2D fp8 weight, got shape={tuple(w_u8.shape)}")
    scale_inv = np.asarray(scale_inv, dtype=np.float32)
    if scale_inv.ndim != 2:
        raise RuntimeError(f"expected 2D scale_inv, got shape={tuple(scale_inv.shape)}")
    rows, cols = w_u8.shape
    if scale_inv.shape != block_grid(rows, cols, block_size):
        raise RuntimeError(
            f"shape mismatch: weight={tuple(w_u8.shape)} scale_inv={tuple(scale_inv.shape)} "
            f"expected_scale_inv={block_grid(rows, cols, block_size)} block_size={block_size}")
    w = decode_e4m3fn(w_u8, ref_quirk=ref_quirk)
    if rows % block_size == 0 and cols % block_size == 0:
        # whole blocks: the same fp32 products, broadcast over a block view (no [r, c] scale copy)
        br, bc = rows // block_size, cols // block_size
        wb = w.reshape(br, block_size, bc, block_size)
        wb *= scale_inv[:, None, :, None]
        return w
    return (w * expand_block_scale(scale_inv, rows, cols, block_size)).astype(np.float32)


def quantize_fp8_blockwise(w: np.ndarray, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """fp32 ``[r, c]`` -> (E4M3FN bytes ``[r, c]``, fp32 ``scale_inv`` ``[ceil(r/b), ceil(c/b)]``).

    Per block: ``s = amax / 448`` (``s = 1`` for an all-zero block), ``q = rne(W / s)``
    clipped to +-448.  All arithmetic is float32, matching the GPU generator in
    ``constellation_b200.synthetic``.
    """
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    br, bc = block_grid(rows, cols, block)
    pad = np.zeros((br * block, bc * block), dtype=np.float32)
    pad[:rows, :cols] = w
    blocks = pad.reshape(br, block, bc, block)
    amax = np.abs(blocks).max(axis=(1, 3)).astype(np.float32)
    s = np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    q = (blocks / s[:, None, :, None]).astype(np.float32)
    q = np.clip(q, -E4M3_MAX, E4M3_MAX)
    codes = encode_e4m3fn_rne(q).reshape(br * block, bc * block)[:rows, :cols]
    return np.ascontiguousarray(codes), s
