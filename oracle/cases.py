"""Seeded synthetic inputs in the shapes of the benchmark configurations (test infrastructure only).

Follows the benchmark's config 0: activations ``N(0, 1)``, RMS-normalised per row and cast
to bf16; router weight ``N(0, 0.02)`` ``[E, H]`` fp32; correction bias ``N(0, 0.01)``;
expert weights ``N(0, 0.02)`` quantized per 128x128 block to E4M3 with fp32
``scale_inv``.  All streams come from ``oracle.detrand`` so a seed pins the data.
"""
from __future__ import annotations

import numpy as np

from . import detrand
from .codec import decode_bf16, encode_bf16_rne
from .fp8 import quantize_fp8_blockwise
from .refbuild import ExpertBytes


def activations(seed: int, T: int, H: int) -> np.ndarray:
    """``[T, H]`` fp32 values that are exactly representable in bf16."""
    x = detrand.normal(seed, (T, H)).astype(np.float32)
    x = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)
    return decode_bf16(encode_bf16_rne(x.astype(np.float32)))


def router(seed: int, E: int, H: int, bias_std: float = 0.01):
    w = detrand.normal(seed * 7919 + 1, (E, H), std=0.02)
    b = detrand.normal(seed * 7919 + 2, (E,), std=bias_std)
    return w, b


def zipf_bias(seed: int, E: int, s: float = 1.2, amp: float = 2.0) -> np.ndarray:
    """Skewed router bias of config 4: ``amp * log-Zipf(s)`` over a seeded expert permutation."""
    perm = detrand.permutation(seed * 31 + 5, E)
    ranks = np.empty(E, dtype=np.float64)
    ranks[perm] = np.arange(1, E + 1)
    return (amp * (-s * np.log(ranks))).astype(np.float32)


def expert(seed: int, H: int, I: int, std: float = 0.02, block: int = 128) -> ExpertBytes:
    base = seed * 104729 + 11
    wu = detrand.normal(base + 1, (I, H), std=std)
    wg = detrand.normal(base + 2, (I, H), std=std)
    wd = detrand.normal(base + 3, (H, I), std=std)
    qu, su = quantize_fp8_blockwise(wu, block)
    qg, sg = quantize_fp8_blockwise(wg, block)
    qd, sd = quantize_fp8_blockwise(wd, block)
    return ExpertBytes(qu, su, qg, sg, qd, sd, block)


def random_fp8_bytes(seed: int, shape, allow_nan: bool = False) -> np.ndarray:
    b = (detrand.splitmix64(seed, int(np.prod(shape))) & np.uint64(0xFF)).astype(np.uint8)
    if not allow_nan:
        b = np.where((b & 0x7F) == 0x7F, b - 1, b).astype(np.uint8)
    return b.reshape(shape)
