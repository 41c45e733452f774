"""The reference-interface mirror (constellation_b200.moe_layer_runtime / fp8_utils) on a GPU.

Tolerances as in test_gpu_parity.py: routing equal on every token (these seeds have no
near-tie), layer outputs within 2e-3 row-wise relative error of the fp32 oracle (bf16
outputs: 1e-2), dequant bit-exact against the reference's own function (golden fixture).
"""
import numpy as np
import pytest
import torch

from oracle import cases
from oracle.expert import DequantExpert

pytestmark = pytest.mark.gpu

E, H, I, G, TG, K = 32, 256, 128, 4, 2, 4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def rowwise_rel(a, ref):
    a = np.atleast_2d(a).astype(np.float64)
    ref = np.atleast_2d(ref).astype(np.float64)
    return float((np.abs(a - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)).max())


def test_dequant_matches_reference_function(dev, golden):
    from constellation_b200.fp8_utils import dequant_fp8_weight_blockwise

    g = golden("dequant_golden")
    for name in ("sq", "ragged", "blk64"):
        w = torch.from_numpy(g[f"{name}__w"]).to(dev)
        s = torch.from_numpy(g[f"{name}__s"]).to(dev)
        out = dequant_fp8_weight_blockwise(w.view(torch.float8_e4m3fn), s, int(g[f"{name}__block"]))
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), g[f"{name}__out"].view(np.uint32))


def test_route_token_real_matches_reference_golden(dev, golden):
    from constellation_b200.moe_layer_runtime import route_token_real

    g = golden("router_golden")
    seed, T, En, Hn, Gn, TGn, Kn = (int(v) for v in g["full__cfg"])
    x = cases.activations(seed, T, Hn)
    w, b = cases.router(seed, En, Hn)
    wt, bt = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
    kw = dict(n_group=Gn, topk_group=TGn, top_k=Kn, norm_topk_prob=True, routed_scaling_factor=2.5,
              scoring_func="sigmoid", topk_method="noaux_tc", n_routed_experts=En, hidden_size=Hn)
    for t in range(T):
        routes, aux = route_token_real(torch.from_numpy(x[t]).to(dev), wt, bt, return_aux=True, **kw)
        assert [e for e, _ in routes] == g["full__topk_idx"][t].tolist()
        np.testing.assert_allclose([v for _, v in routes], g["full__topk_weight"][t], rtol=2e-6)
        for key in ("logits", "group_scores", "selected_group_idx", "topk_idx", "topk_weight", "routes"):
            assert key in aux
    # batched form
    routes_b = route_token_real(torch.from_numpy(x).to(dev), wt, bt, **kw)
    assert [[e for e, _ in r] for r in routes_b] == g["full__topk_idx"].tolist()


def _session(dev, seed=71, T=5):
    from constellation_b200.context import ExpertContext, MoEConfig
    from constellation_b200.moe_layer_runtime import MoESession

    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                    num_experts_per_tok=K)
    ctx = ExpertContext(dev, cfg, n_slots=E + 1, max_tokens=max(T, 8))
    experts = {e: cases.expert(seed * 100 + e, H, I) for e in range(E)}
    for e, b in experts.items():
        ctx.upload_bundle(e, e, b)
    shared = cases.expert(seed * 100 + 99, H, I)
    ctx.upload_bundle(E, -1, shared)
    w, b = cases.router(seed, E, H, bias_std=0.05)
    rc = dict(hidden_size=H, n_routed_experts=E, n_group=G, topk_group=TG, top_k=K, norm_topk_prob=True,
              routed_scaling_factor=2.5, scoring_func="sigmoid", topk_method="noaux_tc")
    s = MoESession(rc, experts_per_layer=E)
    s.add_layer(3, ctx, torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev))
    return s, experts, shared, w, b


def test_run_moe_layer_single_and_batched(dev):
    from constellation_b200.moe_layer_runtime import run_moe_layer
    from oracle.layer import moe_layer

    s, experts, shared, w, b = _session(dev)
    x = cases.activations(72, 5, H)
    ref = moe_layer(x, w, b, {e: DequantExpert(v) for e, v in experts.items()}, None, n_group=G, topk_group=TG,
                    top_k=K)
    xb = torch.from_numpy(x).to(dev, torch.bfloat16)
    out = run_moe_layer(s, xb, 3, return_aux=True)
    assert out["output"].dtype == torch.bfloat16 and out["output"].shape == (5, H)
    assert rowwise_rel(out["output"].float().cpu().numpy(), ref.out_f32) < 1e-2
    one = run_moe_layer(s, xb[2], 3, return_aux=True)
    assert one["output"].shape == (H,)
    assert torch.equal(one["output"], out["output"][2])
    assert one["aux"]["selected_global_expert_ids"] == [3 * E + int(e) for e in ref.route.topk_idx[2]]
    # the reference's 1-D aux keys (server/moe_layer_runtime.py:559-575 with the router's :389-407)
    for key in ("logits", "scores", "group_scores", "selected_group_idx", "group_mask", "topk_weight_pre_norm",
                "weighted_outputs", "combined_pre_cast", "expert_outputs", "resident_local_expert_ids"):
        assert key in one["aux"], key
    assert len(one["aux"]["weighted_outputs"]) == K and len(one["aux"]["expert_outputs"]) == K
    assert rowwise_rel(one["aux"]["combined_pre_cast"], ref.out_f32[2]) < 2e-3


def test_run_topk_moe_layer_and_infer_one_expert(dev):
    from constellation_b200.moe_layer_runtime import infer_one_expert, run_topk_moe_layer

    s, experts, _, _, _ = _session(dev, seed=73)
    x = cases.activations(74, 1, H)[0]
    routes = [(3 * E + 4, 0.7), (3 * E + 9, 1.3)]
    combined, weighted = run_topk_moe_layer(s, torch.from_numpy(x).to(dev, torch.float32), routes)
    ref = 0.7 * DequantExpert(experts[4]).forward(x[None])[0] + 1.3 * DequantExpert(experts[9]).forward(x[None])[0]
    assert rowwise_rel(combined.cpu().numpy(), ref) < 2e-3
    c2, w2, eo = run_topk_moe_layer(s, torch.from_numpy(x).to(dev, torch.float32), routes, return_aux=True)
    assert len(eo) == 2 and eo[0]["output_dtype"] == 1
    assert rowwise_rel(c2.cpu().numpy(), ref) < 2e-3  # fp16 expert outputs, fp32 combine
    r = infer_one_expert(s, 3 * E + 4, x)
    assert r["output_dtype"] == 1 and len(r["output"]) == 2 * H
    with pytest.raises(RuntimeError):
        infer_one_expert(s, 7 * E + 1, x)  # layer not loaded -> not in placements


def test_run_sparse_moe_block_with_residual(dev):
    from constellation_b200.moe_layer_runtime import run_sparse_moe_block
    from oracle.layer import moe_layer

    s, experts, shared, w, b = _session(dev, seed=75, T=6)
    x = cases.activations(76, 6, H)
    resid = cases.activations(77, 6, H)
    ref = moe_layer(x, w, b, {e: DequantExpert(v) for e, v in experts.items()}, DequantExpert(shared), n_group=G,
                    topk_group=TG, top_k=K)
    out = run_sparse_moe_block(s, torch.from_numpy(x).to(dev, torch.bfloat16), 3,
                               residual=torch.from_numpy(resid).to(dev, torch.bfloat16))
    assert rowwise_rel(out.float().cpu().numpy(), ref.out_f32 + resid) < 1e-2


def test_ep_single_rank_equals_fused_layer(dev):
    """world = 1: route -> routed (fp32) -> shared_combine equals the fused layer bit for bit."""
    from constellation_b200.ep import ExpertParallelMoE

    s, _, _, _, _ = _session(dev, seed=78, T=7)
    ctx = s.contexts[3]
    gw = s.backbone_store.layer(3)["router"]["gate_weight"]
    gb = s.backbone_store.layer(3)["router"]["e_score_correction_bias"]
    x = torch.from_numpy(cases.activations(79, 7, H)).to(dev, torch.bfloat16)
    moe = ExpertParallelMoE(ctx, rank=0, world=1, n_routed_experts=E)
    assert torch.equal(moe.forward(x, gw, gb), ctx.moe_layer(x, gw, gb))
