"""Host-side logic that needs no GPU: placement helpers, route validation, combine, config."""
import numpy as np
import pytest
import torch

from constellation_b200 import expert_placement as ep


def test_global_expert_id_round_trip():
    assert ep.make_global_expert_id(3, 17) == 3 * 256 + 17
    assert ep.split_global_expert_id(3 * 256 + 17) == (3, 17)
    assert ep.make_global_expert_id(0, 5, experts_per_layer=8) == 5
    for bad in [(-1, 0), (0, -1), (0, 256)]:
        with pytest.raises(ValueError):
            ep.make_global_expert_id(*bad)
    with pytest.raises(ValueError):
        ep.split_global_expert_id(-5)


def test_allowed_local_ids_and_lookup():
    gids = [ep.make_global_expert_id(2, e) for e in (7, 3, 7, 100)] + [ep.make_global_expert_id(1, 9)]
    assert ep.allowed_local_expert_ids_for_layer(gids, layer_id=2) == [3, 7, 100]
    placements = [{"expert_id": 5, "host": "a", "control_port": 1}, {"expert_id": 2, "host": "a", "control_port": 1},
                  {"expert_id": 9, "host": "b", "control_port": 2}]
    assert ep.find_expert_placement(placements, 9)["host"] == "b"
    with pytest.raises(RuntimeError):
        ep.find_expert_placement(placements, 4)
    g = ep.group_placements_by_control_endpoint(placements)
    assert [p["expert_id"] for p in g[("a", 1)]] == [2, 5]
    assert ep.ep_owner_rank(200, 256, 8) == 6


def test_route_validation_and_normalisation():
    from constellation_b200.moe_layer_runtime import normalize_routes, validate_routes

    validate_routes([(1, 0.5), (2, 0.25)])
    for bad in ([], [(1, 0.5), (1, 0.2)], [(1, -0.1)]):
        with pytest.raises(RuntimeError):
            validate_routes(bad)
    assert normalize_routes([(1, 1.0), (2, 3.0)]) == [(1, 0.25), (2, 0.75)]
    with pytest.raises(RuntimeError):
        normalize_routes([(1, 0.0)])


def test_combine_outputs_torch_fp32_sum():
    from constellation_b200.moe_layer_runtime import combine_outputs_torch

    ys = [(1, 0.5, np.ones(4, np.float32)), (2, 2.0, np.arange(4, dtype=np.float32))]
    out = combine_outputs_torch(ys, out_dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert out.float().tolist() == [0.5, 2.5, 4.5, 6.5]
    with pytest.raises(RuntimeError):
        combine_outputs_torch([], out_dtype=torch.float32)


def test_route_token_real_argument_errors_match_reference():
    from constellation_b200.moe_layer_runtime import route_token_real

    kw = dict(n_group=8, topk_group=4, top_k=8, norm_topk_prob=True, routed_scaling_factor=2.5,
              scoring_func="sigmoid", topk_method="noaux_tc", n_routed_experts=256, hidden_size=64)
    w = torch.zeros(256, 64)
    b = torch.zeros(256)
    with pytest.raises(RuntimeError):
        route_token_real(torch.zeros(64), w, b, **{**kw, "scoring_func": "softmax"})
    with pytest.raises(TypeError):
        route_token_real([0.0] * 64, w, b, **kw)
    with pytest.raises(TypeError):
        route_token_real(torch.zeros(64, dtype=torch.bfloat16), w, b, **kw)
    with pytest.raises(RuntimeError):
        route_token_real(torch.zeros(32), w, b, **kw)
    with pytest.raises(RuntimeError):
        route_token_real(torch.zeros(64), w, b, **{**kw, "topk_group": 9})
    with pytest.raises(RuntimeError):  # CPU weights: the CUDA router is the only implementation
        route_token_real(torch.zeros(64), w, b, **kw)


def test_synthetic_quantizer_matches_oracle():
    from constellation_b200.synthetic import quantize_blockwise
    from oracle import cases
    from oracle.fp8 import quantize_fp8_blockwise

    w = cases.detrand.normal(5, (256, 384), std=0.02)
    q_ref, s_ref = quantize_fp8_blockwise(w)
    q, s = quantize_blockwise(torch.from_numpy(w))
    np.testing.assert_array_equal(q.numpy(), q_ref)
    np.testing.assert_array_equal(s.numpy(), s_ref)


def test_dequant_cpu_input_needs_cuda():
    from constellation_b200.fp8_utils import dequant_fp8_weight_blockwise

    with pytest.raises(RuntimeError):
        dequant_fp8_weight_blockwise(torch.zeros(4, 4, dtype=torch.uint8), torch.ones(2, 2))  # bad grid


def test_moe_config_from_the_reference_router_config():
    """``MoEConfig.from_router_config`` reads the dict of ``DeepSeekModelLoader.router_config``
    (server/deepseek_model_loader.py:66-81) and rejects the routers the kernels do not run."""
    from constellation_b200.context import MoEConfig

    rc = {"n_group": 8, "topk_group": 4, "top_k": 8, "norm_topk_prob": True, "routed_scaling_factor": 2.5,
          "scoring_func": "sigmoid", "topk_method": "noaux_tc", "n_routed_experts": 256, "hidden_size": 7168}
    assert MoEConfig.from_router_config(rc, inter=2048) == MoEConfig()
    with pytest.raises(RuntimeError, match="scoring_func"):
        MoEConfig.from_router_config({**rc, "scoring_func": "softmax"}, inter=2048)
    with pytest.raises(RuntimeError, match="topk_method"):
        MoEConfig.from_router_config({**rc, "topk_method": "greedy"}, inter=2048)


def test_replica_choice_balances_skewed_routes():
    """choose_replicas / rows_per_rank (constellation_b200.ep): a Zipf-like route skew that
    loads one rank, balanced by replicating the hot experts; each row counted exactly once."""
    import numpy as np

    from constellation_b200 import ep

    rng = np.random.default_rng(7)
    W, E, T, K = 4, 32, 256, 4
    p = 1.0 / np.arange(1, E + 1) ** 1.5
    idx = np.stack([rng.choice(E, size=K, replace=False, p=p / p.sum()) for _ in range(T)])
    base = ep.rows_per_rank(idx, W, E)
    assert sum(base) == T * K + T  # every route plus one shared row per token
    assert max(base) / (sum(base) / W) > 1.5  # experts 0-7 all live on rank 0
    reps = ep.choose_replicas(idx, W, E, target=1.1)
    bal = ep.rows_per_rank(idx, W, E, reps)
    assert sum(bal) == sum(base)
    assert max(bal) / (sum(bal) / W) <= 1.1
    assert reps == sorted(reps) and 0 in reps
    assert ep.choose_replicas(idx, 1, E) == []
