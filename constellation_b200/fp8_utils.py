"""FP8 helpers with the interface of the reference's ``server/fp8_utils.py``.

``dequant_fp8_weight_blockwise`` keeps the reference's signature, shape checks and
errors (``server/fp8_utils.py:4-25``) and computes on the GPU with the library's
dequant kernel (``cst_dequant_fp8``); the result is bit-identical to the reference's
block loop (``:27-39``).  CPU inputs are copied to the current CUDA device and the
result is returned on the input's device; there is no CPU implementation.
"""
from __future__ import annotations

import torch


def dequant_fp8_weight_blockwise(weight_fp8: torch.Tensor, scale_inv: torch.Tensor,
                                 block_size: int = 128) -> torch.Tensor:
    if weight_fp8.ndim != 2:
        raise RuntimeError(f"expected 2D fp8 weight, got shape={tuple(weight_fp8.shape)}")
    if scale_inv.ndim != 2:
        raise RuntimeError(f"expected 2D scale_inv, got shape={tuple(scale_inv.shape)}")
    rows, cols = weight_fp8.shape
    br, bc = scale_inv.shape
    expected_br = (rows + block_size - 1) // block_size
    expected_bc = (cols + block_size - 1) // block_size
    if br != expected_br or bc != expected_bc:
        raise RuntimeError(
            f"shape mismatch: weight={tuple(weight_fp8.shape)} scale_inv={tuple(scale_inv.shape)} "
            f"expected_scale_inv=({expected_br}, {expected_bc}) block_size={block_size}")
    from . import _lib

    home = weight_fp8.device
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    w = weight_fp8
    if w.dtype == torch.float8_e4m3fn:
        w = w.view(torch.uint8)
    if w.dtype != torch.uint8:
        raise TypeError(f"weight must be float8_e4m3fn (or its uint8 bytes), got {weight_fp8.dtype}")
    w = w.to(dev).contiguous()
    s = scale_inv.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.cst_dequant_fp8(w.data_ptr(), s.data_ptr(), rows, cols, int(block_size), out.data_ptr(),
                                            torch.cuda.current_stream(dev).cuda_stream))
    return out if home.type == "cuda" else out.to(home)
