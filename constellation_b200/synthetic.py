"""Seeded synthetic DeepSeek-V3 MoE layers generated on the GPU (benchmark inputs).

The benchmark's config 0 defines the data: activations ``N(0, 1)`` RMS-normalised per row and
cast to bf16; router weight ``N(0, 0.02)`` ``[E, H]`` fp32 and correction bias
``N(0, 0.01)``; expert weights ``N(0, 0.02)`` quantized per 128x128 block with
``s = amax / 448``, ``q = e4m3fn(W / s)`` (saturating) and ``s`` kept as ``scale_inv``
-- the format ``dequant_fp8_weight_blockwise`` (server/fp8_utils.py:4-39) consumes.
There is no public dataset or checkpoint for this path; real DeepSeek-V3.1 weights are
not available, so every benchmark number is on this synthetic data.

Everything here runs as plain torch ops on the target device (data preparation, not the
measured path).
"""
from __future__ import annotations

import torch

# Seeds of the synthetic tensors.  Layer ``l`` of a stack (``l = 0`` for the one-layer
# workloads): routed expert ``e`` is seeded ``1000 (l + 1) + e``, the shared expert
# ``1000 (l + 1) + 999``, the router weight and bias ``7 + 13 l``, the prenorm weight
# ``100 + l``; the activations ``11``.  Each tensor set has its own generator, so one
# expert can be regenerated alone (the parity checks rebuild only the experts they need).
ACTIVATION_SEED = 11


def expert_seed(expert: int, layer: int = 0) -> int:
    """Seed of routed expert ``expert`` of stacked layer ``layer`` (``expert < 0``: the shared one)."""
    return 1000 * (layer + 1) + (999 if expert < 0 else int(expert))


def router_seed(layer: int = 0) -> int:
    return 7 + 13 * layer


def norm_seed(layer: int) -> int:
    return 100 + layer


def quantize_blockwise(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``[r, c]`` (multiples of ``block``) -> (uint8 E4M3FN codes, fp32 scale_inv grid)."""
    r, c = w.shape
    if r % block or c % block:
        raise ValueError("quantize_blockwise needs dimensions that are multiples of the block")
    blocks = w.float().reshape(r // block, block, c // block, block)
    amax = blocks.abs().amax(dim=(1, 3))
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (blocks / s[:, None, :, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.reshape(r, c).view(torch.uint8).contiguous(), s.contiguous()


class SyntheticExpert:
    """The six tensors of one expert in the reference upload format (on ``device``)."""

    def __init__(self, w_up, s_up, w_gate, s_gate, w_down, s_down, block: int = 128):
        self.w_up, self.s_up = w_up, s_up
        self.w_gate, self.s_gate = w_gate, s_gate
        self.w_down, self.s_down = w_down, s_down
        self.block = block


    def host(self) -> "SyntheticExpert":
        """numpy copies of the six tensors (what a CPU checker reads)."""
        t = [v.cpu().numpy() for v in (self.w_up, self.s_up, self.w_gate, self.s_gate, self.w_down, self.s_down)]
        return SyntheticExpert(*t, block=self.block)


def make_expert(hidden: int, inter: int, *, seed: int, device, std: float = 0.02) -> SyntheticExpert:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    out = []
    for shape in ((inter, hidden), (inter, hidden), (hidden, inter)):
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)
        out.extend(quantize_blockwise(w))
        del w
    return SyntheticExpert(*out)


def make_router(hidden: int, n_experts: int, *, seed: int, device, bias_std: float = 0.01):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    w = torch.randn((n_experts, hidden), generator=g, device=device, dtype=torch.float32).mul_(0.02)
    b = torch.randn((n_experts,), generator=g, device=device, dtype=torch.float32).mul_(bias_std)
    return w.contiguous(), b.contiguous()


def zipf_bias(n_experts: int, *, seed: int, device, s: float = 1.2, amp: float = 2.0) -> torch.Tensor:
    """Config 4's skewed bias: ``amp * log-Zipf(s)`` over a seeded permutation of the experts."""
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    perm = torch.randperm(n_experts, generator=g)
    ranks = torch.empty(n_experts, dtype=torch.float64)
    ranks[perm] = torch.arange(1, n_experts + 1, dtype=torch.float64)
    return (amp * (-s * torch.log(ranks))).to(torch.float32).to(device)


def make_activations(T: int, hidden: int, *, seed: int, device, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    x = torch.randn((T, hidden), generator=g, device=device, dtype=torch.float32)
    x = x * torch.rsqrt(x.pow(2).mean(dim=1, keepdim=True) + 1e-6)
    return x.to(dtype).contiguous()


def rms_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(x.dtype)
