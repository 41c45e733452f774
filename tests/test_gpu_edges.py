"""Edge cases of the layer entry points on one GPU: empty batches through every call, the
device packer at its one-CTA limit (2048 routes) and one token past it, T at and past the
context's max_tokens, and top_k below the model's (the ``top_k`` argument of
``route_token_real``, server/moe_layer_runtime.py:232-408), each against the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import cases, router
from oracle.expert import DequantExpert
from oracle.layer import moe_layer

pytestmark = pytest.mark.gpu

E, H, I, G, TG, K = 16, 256, 128, 4, 2, 4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def setup(dev, seed, max_tokens):
    from constellation_b200.context import ExpertContext, MoEConfig

    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                    num_experts_per_tok=K)
    w, b = cases.router(seed, E, H, bias_std=0.05)
    experts = {e: cases.expert(1000 * seed + e, H, I) for e in range(E)}
    sh = cases.expert(1000 * seed + 999, H, I)
    ctx = ExpertContext(dev, cfg, n_slots=E + 1, max_tokens=max_tokens)
    for e in range(E):
        ctx.upload_bundle(e, e, experts[e])
    ctx.upload_bundle(E, -1, sh)
    de = {e: DequantExpert(v) for e, v in experts.items()}
    return ctx, w, b, de, DequantExpert(sh)


def test_empty_batch_is_a_no_op(dev):
    """A [0, H] CUDA tensor has a null data pointer: every call returns an empty result;
    the expert request keeps the worker's answer to batch 0 (backend failure)."""
    from constellation_b200._lib import CST_ERR_BACKEND, CstError
    from constellation_b200.context import rms_norm

    ctx, w, b, de, sh = setup(dev, 350, 8)
    wt, bt = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
    x0 = torch.empty((0, H), dtype=torch.bfloat16, device=dev)
    idx, wts = ctx.route(x0, wt, bt)
    assert idx.shape == (0, K) and wts.shape == (0, K)
    assert ctx.moe_layer(x0, wt, bt).shape == (0, H)
    assert ctx.moe_layer(x0, wt, bt, residual=x0, out_dtype=torch.float32).shape == (0, H)
    assert ctx.moe_routed(x0, idx, wts, add_shared=True).shape == (0, H)
    assert ctx.grouped_ffn(x0, torch.empty(0, dtype=torch.int32, device=dev)).shape == (0, H)
    assert ctx.shared_combine(x0).shape == (0, H)
    assert ctx.cast_extra(torch.empty((0, H), dtype=torch.float32, device=dev)).shape == (0, H)
    assert rms_norm(x0).shape == (0, H)
    with pytest.raises(CstError) as ei:
        ctx.expert_forward(3, x0)
    assert ei.value.code == CST_ERR_BACKEND
    # the context still serves a batch afterwards
    check_layer(ctx, cases.activations(351, 5, H), w, b, de, sh, dev)


def check_layer(ctx, x, w, b, de, sh, dev, top_k=K):
    args = (torch.from_numpy(x).to(dev, torch.bfloat16), torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev))
    out, idx, _ = ctx.moe_layer(*args, top_k=top_k, return_routes=True, out_dtype=torch.float32)
    ref = moe_layer(x, w, b, de, sh, n_group=G, topk_group=TG, top_k=top_k)
    _, _, logits, _ = ctx.route(*args, top_k=top_k, return_aux=True)
    c = router.compare_routes(idx.cpu().numpy(), ref.route.topk_weight, x, w, b, dev_logits=logits.cpu().numpy(),
                              n_group=G, topk_group=TG, top_k=top_k)
    assert c["unexplained"] == 0, c
    ok = np.all(idx.cpu().numpy() == ref.route.topk_idx, axis=1)
    got = out.cpu().numpy()[ok]
    rel = np.abs(got - ref.out_f32[ok]).max(axis=1) / np.abs(ref.out_f32[ok]).max(axis=1)
    assert float(rel.max()) < 2e-3
    return out


@pytest.mark.parametrize("T", [512, 513])
def test_packer_one_cta_limit(dev, T):
    """512 tokens x top-4 = 2048 routes is the largest batch the one-CTA counting sort takes;
    513 goes to the three-launch multi-CTA sort.  Both must give the oracle's layer."""
    ctx, w, b, de, sh = setup(dev, 300 + T, T)
    x = cases.activations(310 + T, T, H)
    out = check_layer(ctx, x, w, b, de, sh, dev)
    # bit-stable on repeat
    again = ctx.moe_layer(torch.from_numpy(x).to(dev, torch.bfloat16), torch.from_numpy(w).to(dev),
                          torch.from_numpy(b).to(dev), out_dtype=torch.float32)
    assert torch.equal(out, again)


@pytest.mark.parametrize("top_k", [1, 2, 3])
def test_top_k_below_the_model(dev, top_k):
    ctx, w, b, de, sh = setup(dev, 320 + top_k, 40)
    x = cases.activations(330 + top_k, 40, H)
    check_layer(ctx, x, w, b, de, sh, dev, top_k=top_k)


def test_max_tokens_is_inclusive(dev):
    from constellation_b200._lib import CST_ERR_INVALID_ARG, CstError

    ctx, w, b, de, sh = setup(dev, 340, 8)
    check_layer(ctx, cases.activations(341, 8, H), w, b, de, sh, dev)
    x9 = torch.from_numpy(cases.activations(342, 9, H)).to(dev, torch.bfloat16)
    with pytest.raises(CstError) as ei:
        ctx.moe_layer(x9, torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev))
    assert ei.value.code == CST_ERR_INVALID_ARG


def test_own_tokens_only_experts_serve_the_own_range():
    """Experts marked own-tokens-only (replicated hot experts under expert parallelism) get
    rows only for tokens inside the call's own-token range, like the shared expert; the
    others serve every token.  Checked through cst_moe_routed_range against the oracle's
    per-route outputs, and unmarking restores the full layer."""
    T, lo, hi = 24, 6, 15
    ctx, w, b, de, sh = setup(dev_or_skip(), 360, T)
    dev = ctx.device
    x = cases.activations(361, T, H)
    xt = torch.from_numpy(x).to(dev, torch.bfloat16)
    idx, wts = ctx.route(xt, torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev))
    marked = (0, 3, 9)
    for e in marked:
        ctx.set_own_tokens_only(e)
    out = ctx.moe_routed_range(xt, idx, wts, lo, hi, out_dtype=torch.float32).cpu().numpy()
    xb = xt.float().cpu().numpy()
    ih, wh = idx.cpu().numpy(), wts.cpu().numpy()
    ref = np.zeros((T, H), np.float32)
    for t in range(T):
        inside = lo <= t < hi
        for k in range(K):
            e = int(ih[t, k])
            if e in marked and not inside:
                continue
            ref[t] += wh[t, k] * de[e].forward(xb[t:t + 1])[0]
        if inside:
            ref[t] += sh.forward(xb[t:t + 1])[0]
    rel = np.abs(out - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)
    assert float(rel.max()) < 2e-3, rel
    for e in marked:
        ctx.set_own_tokens_only(e, False)
    full = ctx.moe_routed_range(xt, idx, wts, 0, T, out_dtype=torch.float32)
    lay = ctx.moe_layer(xt, torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev), out_dtype=torch.float32)
    assert torch.equal(full, lay)


def dev_or_skip():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
