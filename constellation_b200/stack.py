"""Stacked MoE layers over one token batch (the sparse-layer glue around the hot path).

Replaces the per-layer loop of the reference's sparse layer
(``server/full_model_runtime.py:173-379``) for a decode step through many MoE layers with
no attention in between: for each layer ``l``

    xn = rms_norm(h, norm_weight_l, eps)          # :271-276, cst_rmsnorm
    h  = h + routed_l(xn) + shared_l(xn)          # :348-355, residual fused into the last cast

with the whole batch at once (no per-token loop, ``:317-334``).  Each layer has its own
expert context and its own router weights; under expert parallelism every layer runs the
exchange of ``ExpertParallelMoE`` (one process per GPU, NCCL).  Everything is stream
ordered and can be captured in one CUDA graph (all-gather mode).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .context import rms_norm
from .ep import ExpertParallelMoE


@dataclass
class StackLayer:
    """One layer: expert compute (an ``ExpertContext``), router weight ``[E, H]`` fp32,
    correction bias ``[E]`` fp32 and the prenorm weight ``[H]`` fp32 (None: ones)."""

    compute: object
    gate_weight: torch.Tensor
    bias: torch.Tensor
    norm_weight: torch.Tensor | None = None


class MoEStack:
    def __init__(self, layers: list[StackLayer], *, rank: int = 0, world: int = 1, n_routed_experts: int = 256,
                 group=None, mode: str = "allgather", eps: float = 1e-6, norm=None, p2p_tl_cap: int | None = None):
        if not layers:
            raise ValueError("MoEStack needs at least one layer")
        self.layers = layers
        self.eps = float(eps)
        self.norm = norm or rms_norm
        self.moe = [ExpertParallelMoE(l.compute, rank=rank, world=world, n_routed_experts=n_routed_experts,
                                      group=group, mode=mode, p2p_tl_cap=p2p_tl_cap) for l in layers]

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """``h [T_local, H]`` (this rank's tokens) -> the hidden state after every layer, same dtype."""
        for layer, moe in zip(self.layers, self.moe):
            xn = self.norm(h, layer.norm_weight, self.eps)
            h = moe.forward(xn, layer.gate_weight, layer.bias, residual=h, out_dtype=h.dtype)
        return h

    def close(self) -> None:
        """Release every layer's peer-exchange buffers (p2p mode; every rank, after its last
        forward, behind a barrier)."""
        for moe in self.moe:
            moe.close()
