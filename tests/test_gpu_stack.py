"""RMSNorm (cst_rmsnorm) and the stacked-layer driver on one GPU against the oracle.

The prenorm is torch.nn.functional.rms_norm(h, (H,), weight, 1e-6)
(server/full_model_runtime.py:271-276); the stack is prenorm -> MoE -> residual per layer
(:348-355) with every tensor handed between layers in bf16 (oracle.layer.moe_stack).
"""
import numpy as np
import pytest
import torch

from oracle import cases
from oracle.expert import DequantExpert
from oracle.layer import moe_stack

pytestmark = pytest.mark.gpu

E, H, I, G, TG, K = 16, 256, 128, 4, 2, 4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("dt,weighted", [(torch.bfloat16, True), (torch.bfloat16, False), (torch.float16, True),
                                         (torch.float32, True)])
def test_rms_norm_matches_fp32_reference(dev, dt, weighted):
    from constellation_b200.context import rms_norm

    T, Hn = 37, 7168
    g = torch.Generator(device="cpu").manual_seed(5)
    x = (torch.randn((T, Hn), generator=g) * 3.0).to(dev, dt)
    w = (1.0 + 0.1 * torch.randn((Hn,), generator=g)).to(dev) if weighted else None
    y = rms_norm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + 1e-6)
    if weighted:
        ref = ref * w
    if dt == torch.float32:
        torch.testing.assert_close(y, ref, rtol=2e-6, atol=1e-6)
    else:
        # one rounding of the fp32 result: half an ulp of the output type (2^-9 bf16,
        # 2^-12 fp16 relative), with room for the fp32 reduction-order difference
        tol = 2 ** -8 if dt == torch.bfloat16 else 2 ** -10
        assert ((y.float() - ref).abs() <= ref.abs() * tol + 1e-6).all()
        # and torch's own rms_norm on the same input within one ulp
        tr = torch.nn.functional.rms_norm(x, (Hn,), w.to(dt) if weighted else None, 1e-6)
        assert ((y.float() - tr.float()).abs() <= tr.float().abs() * 2 ** -6 + 1e-6).all()


def test_rms_norm_in_place_and_rejects_bad_shape(dev):
    from constellation_b200 import _lib
    from constellation_b200.context import rms_norm

    x = torch.randn((4, 256), device=dev).to(torch.bfloat16)
    ref = rms_norm(x.clone())
    rms_norm(x, out=x)
    assert torch.equal(x, ref)
    bad = torch.zeros((2, 12), device=dev, dtype=torch.bfloat16)
    rc = _lib.lib.cst_rmsnorm(bad.data_ptr(), 2, 2, 12, None, 1e-6, bad.data_ptr(), 2, None)
    assert rc == _lib.CST_ERR_INVALID_ARG


def test_moe_stack_three_layers_vs_oracle(dev):
    from constellation_b200.context import ExpertContext, MoEConfig
    from constellation_b200.stack import MoEStack, StackLayer

    T, L = 20, 3
    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                    num_experts_per_tok=K)
    layers, ref_layers = [], []
    for l in range(L):
        w, b = cases.router(170 + l, E, H, bias_std=0.05)
        ex = {e: cases.expert(7000 + 100 * l + e, H, I) for e in range(E)}
        sh = cases.expert(7099 + 100 * l, H, I)
        nw = (1.0 + 0.1 * cases.activations(180 + l, 1, H)[0]).astype(np.float32)
        ctx = ExpertContext(dev, cfg, n_slots=E + 1, max_tokens=T)
        for e in range(E):
            ctx.upload_bundle(e, e, ex[e])
        ctx.upload_bundle(E, -1, sh)
        layers.append(StackLayer(ctx, torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev),
                                 torch.from_numpy(nw).to(dev)))
        ref_layers.append((w, b, {e: DequantExpert(v) for e, v in ex.items()}, DequantExpert(sh), nw))
    stack = MoEStack(layers, n_routed_experts=E)
    h0 = cases.activations(190, T, H)
    out = stack.forward(torch.from_numpy(h0).to(dev, torch.bfloat16))
    ref = moe_stack(h0, ref_layers, n_group=G, topk_group=TG, top_k=K)
    got = out.float().cpu().numpy()
    rel = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert float(rel.max()) < 1e-2
    # bit-stable on repeat
    assert torch.equal(stack.forward(torch.from_numpy(h0).to(dev, torch.bfloat16)), out)
