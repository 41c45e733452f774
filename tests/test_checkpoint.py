"""DeepSeek checkpoint ingest (``constellation_b200.checkpoint``) on a synthetic checkpoint.

``write_checkpoint`` below writes a small DeepSeek-style checkpoint -- ``config.json``,
``model.safetensors.index.json`` and two safetensors shards written by the ``safetensors``
package itself (not by the reader under test), with the routed experts, the shared expert,
the router weight (bf16) and its correction bias of two layers in DeepSeek's tensor names
and ``*_scale_inv`` block scales.  The CPU tests read it back and compare the names, the
index resolution and the preload manifest with the reference's own loader and coordinator
(server/deepseek_model_loader.py, server/coordinator.py:413-488) where the reference tree
is present; the GPU test uploads a layer from it and checks the layer against the oracle.
"""
import json

import numpy as np
import pytest
import torch

from oracle import cases

H, I, E, G, TG, K, LAYERS = 256, 128, 16, 4, 2, 4, 2


def _fp8(e):
    return torch.from_numpy(np.ascontiguousarray(e)).view(torch.float8_e4m3fn)


def write_checkpoint(root, *, layers=LAYERS, experts=E, hidden=H, inter=I):
    """The synthetic checkpoint; returns {(layer, expert or -1): bundle} and {layer: (gate, bias)}."""
    from safetensors.torch import save_file

    bundles, routers = {}, {}
    shard_tensors = [{}, {}]
    for layer in range(layers):
        shard = shard_tensors[layer % 2]
        for e in list(range(experts)) + [-1]:
            b = cases.expert(5000 + 100 * layer + (99 if e < 0 else e), hidden, inter)
            bundles[(layer, e)] = b
            base = (f"model.layers.{layer}.mlp.shared_experts" if e < 0
                    else f"model.layers.{layer}.mlp.experts.{e}")
            for proj, w, s in (("up_proj", b.w_up, b.s_up), ("gate_proj", b.w_gate, b.s_gate),
                               ("down_proj", b.w_down, b.s_down)):
                shard[f"{base}.{proj}.weight"] = _fp8(w)
                shard[f"{base}.{proj}.weight_scale_inv"] = torch.from_numpy(np.ascontiguousarray(s))
        gw, gb = cases.router(6000 + layer, experts, hidden, bias_std=0.05)
        gw16 = torch.from_numpy(gw).to(torch.bfloat16)
        routers[layer] = (gw16.float().numpy(), gb)
        shard[f"model.layers.{layer}.mlp.gate.weight"] = gw16
        shard[f"model.layers.{layer}.mlp.gate.e_score_correction_bias"] = torch.from_numpy(gb)
    weight_map = {}
    for i, tensors in enumerate(shard_tensors):
        name = f"model-{i + 1:05d}-of-00002.safetensors"
        save_file(tensors, str(root / name))
        weight_map.update({k: name for k in tensors})
    (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    (root / "config.json").write_text(json.dumps({
        "hidden_size": hidden, "moe_intermediate_size": inter, "n_routed_experts": experts, "n_group": G,
        "topk_group": TG, "num_experts_per_tok": K, "norm_topk_prob": True, "routed_scaling_factor": 2.5,
        "scoring_func": "sigmoid", "topk_method": "noaux_tc"}))
    return bundles, routers


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    pytest.importorskip("safetensors")
    root = tmp_path_factory.mktemp("deepseek_ckpt")
    bundles, routers = write_checkpoint(root)
    return root, bundles, routers


def _reference_modules():
    from oracle import refbuild

    root = refbuild.reference_root()
    if root is None:
        pytest.skip("the reference tree is not present")
    import sys

    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    try:
        from server import coordinator, deepseek_model_loader
    except Exception as exc:  # an import the reference needs is missing here
        pytest.skip(f"reference server modules do not import: {exc}")
    return coordinator, deepseek_model_loader


def test_reads_tensors_and_router(ckpt):
    from constellation_b200.checkpoint import DeepseekCheckpoint

    root, bundles, routers = ckpt
    c = DeepseekCheckpoint(root)
    assert c.router_config()["n_routed_experts"] == E and c.router_config()["top_k"] == K
    for (layer, e), b in bundles.items():
        got = c.expert_bundle(layer, None if e < 0 else e)
        for k_got, k_ref in (("w_up", "w_up"), ("w_up_scale", "s_up"), ("w_gate", "w_gate"),
                             ("w_gate_scale", "s_gate"), ("w_down", "w_down"), ("w_down_scale", "s_down")):
            np.testing.assert_array_equal(np.asarray(got[k_got]), getattr(b, k_ref))
    for layer, (gw, gb) in routers.items():
        w, bias = c.router_tensors(layer)
        np.testing.assert_array_equal(w, gw)
        np.testing.assert_array_equal(bias, gb)
    with pytest.raises(KeyError):
        c.resolve_deepseek_tensor(0, E, "w_up")
    with pytest.raises(ValueError):
        c.resolve_deepseek_tensor(0, 0, "w_mid")


def test_names_index_and_manifest_match_the_reference(ckpt):
    from constellation_b200.checkpoint import DeepseekCheckpoint, deepseek_tensor_name

    coordinator, dml = _reference_modules()
    root, _, _ = ckpt
    for layer, e, kind in ((0, 0, "w_up"), (3, 255, "w_gate"), (60, 17, "w_down")):
        assert deepseek_tensor_name(layer, e, kind) == dml.deepseek_tensor_name(layer, e, kind)
    ref = dml.DeepseekModelLoader(str(root))
    ours = DeepseekCheckpoint(root)
    assert ours.weight_map() == ref.weight_map()
    assert ours.resolve_deepseek_scale_tensor(1, 5, "w_down") == ref.resolve_deepseek_scale_tensor(1, 5, "w_down")
    placements = [{"expert_id": gid, "host": h, "control_port": p}
                  for gid, h, p in ((E + 3, "b", 1), (2, "a", 2), (5, "a", 1), (E + 0, "a", 1), (1, "b", 1))]

    class _Coord:  # the method reads only its arguments
        pass

    want = coordinator.Coordinator.build_preload_manifest(_Coord(), ref, experts_per_layer=E, placements=placements) \
        if hasattr(coordinator, "Coordinator") else None
    if want is None:
        pytest.skip("the reference coordinator class is not importable as Coordinator")
    got = ours.build_preload_manifest(placements, experts_per_layer=E)
    assert [b.expert_id for b in got] == [b.expert_id for b in want]
    for g, w in zip(got, want):
        assert [(t.tensor_kind_name, t.tensor_order, t.tensor_name, t.shard_path) for t in g.tensors] == \
            [(t.tensor_kind_name, t.tensor_order, t.tensor_name, t.shard_path) for t in w.tensors]


def test_reference_loader_dequantizes_what_we_upload(ckpt):
    """The reference's own loader reads the synthetic shards (fp32 dequant through its
    dequant_fp8_weight_blockwise) to the same weights the oracle derives from our bundle."""
    from constellation_b200.checkpoint import DeepseekCheckpoint
    from oracle.fp8 import dequant_fp8_weight_blockwise

    _, dml = _reference_modules()
    root, _, _ = ckpt
    ref = dml.DeepseekModelLoader(str(root))
    ours = DeepseekCheckpoint(root).expert_bundle(1, 7)
    w_up, _, w_down = ref.load_routed_expert_triplet_fp32(1, 7)
    np.testing.assert_array_equal(w_up.numpy(), dequant_fp8_weight_blockwise(np.asarray(ours["w_up"]),
                                                                              np.asarray(ours["w_up_scale"])))
    np.testing.assert_array_equal(w_down.numpy(), dequant_fp8_weight_blockwise(np.asarray(ours["w_down"]),
                                                                               np.asarray(ours["w_down_scale"])))


@pytest.mark.gpu
def test_layer_uploaded_from_checkpoint_vs_oracle(ckpt):
    from constellation_b200.checkpoint import DeepseekCheckpoint
    from constellation_b200.context import ExpertContext, MoEConfig
    from oracle import router
    from oracle.expert import DequantExpert
    from oracle.layer import moe_layer

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    root, bundles, routers = ckpt
    dev = torch.device("cuda", 0)
    c = DeepseekCheckpoint(root)
    rc = c.router_config()
    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=rc["n_routed_experts"],
                    n_group=rc["n_group"], topk_group=rc["topk_group"], num_experts_per_tok=rc["top_k"])
    layer = 1
    T = 24
    ctx = ExpertContext(dev, cfg, n_slots=E + 1, max_tokens=T)
    try:
        placed = c.upload_layer(ctx, layer)
        assert placed[-1] == E and sorted(k for k in placed if k >= 0) == list(range(E))
        gw, gb = c.router_tensors(layer)
        x = cases.activations(6100, T, H)
        xt = torch.from_numpy(x).to(dev, torch.bfloat16)
        out, idx, _ = ctx.moe_layer(xt, torch.from_numpy(gw).to(dev), torch.from_numpy(gb).to(dev),
                                    return_routes=True, out_dtype=torch.float32)
        torch.cuda.synchronize(dev)
        xb = xt.float().cpu().numpy()
        de = {e: DequantExpert(bundles[(layer, e)]) for e in range(E)}
        ref = moe_layer(xb, gw, gb, de, DequantExpert(bundles[(layer, -1)]), n_group=G, topk_group=TG, top_k=K)
        c_r = router.compare_routes(idx.cpu().numpy(), ref.route.topk_weight, xb, gw, gb, n_group=G,
                                    topk_group=TG, top_k=K)
        assert c_r["mismatched"] == 0, c_r
        got = out.cpu().numpy()
        rel = (np.abs(got - ref.out_f32).max(axis=1) / np.abs(ref.out_f32).max(axis=1)).max()
        assert rel < 2e-3, rel
    finally:
        ctx.close()
