"""fp32 SwiGLU expert on block-dequantized FP8 weights (CPU oracle; test infrastructure only).

Restates ``run_one_expert_reference`` (``server/moe_layer_runtime.py:581-611``): the
weights are dequantized with ``dequant_fp8_weight_blockwise`` (``server/fp8_utils.py:4``)
and then ``up = x @ Wu.T``, ``gate = x @ Wg.T``, ``fused = up * silu(gate)``,
``y = fused @ Wd.T`` in fp32 (``:604-609``).  The same function serves the shared
expert (``server/deepseek_full_model_executor.py:296-299``), whose weights the
benchmark configuration quantizes like the routed ones.
"""
from __future__ import annotations

import numpy as np

from .fp8 import dequant_fp8_weight_blockwise


def silu_f32(g: np.ndarray) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    return (g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))).astype(np.float32)


class DequantExpert:
    """Dequantized fp32 weights of one expert (cache them: dequant is the slow part)."""

    def __init__(self, e, *, ref_quirk: bool = False):
        b = e.block
        self.w_up = dequant_fp8_weight_blockwise(e.w_up, e.s_up, b, ref_quirk=ref_quirk)
        self.w_gate = dequant_fp8_weight_blockwise(e.w_gate, e.s_gate, b, ref_quirk=ref_quirk)
        self.w_down = dequant_fp8_weight_blockwise(e.w_down, e.s_down, b, ref_quirk=ref_quirk)

    def forward(self, x: np.ndarray, *, return_h: bool = False):
        x = np.atleast_2d(np.asarray(x, dtype=np.float32))
        up = x @ self.w_up.T
        gate = x @ self.w_gate.T
        fused = (up * silu_f32(gate)).astype(np.float32)
        y = (fused @ self.w_down.T).astype(np.float32)
        return (y, fused) if return_h else y


def expert_forward(e, x: np.ndarray, *, ref_quirk: bool = False) -> np.ndarray:
    return DequantExpert(e, ref_quirk=ref_quirk).forward(x)
