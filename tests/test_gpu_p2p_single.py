"""The peer-exchange kernels (cst_moe_routed_push / cst_reduce_pushed) on one GPU, through a
one-rank cst_peer_set filled by hand over a torch buffer -- the way a C++ host that owns its
own mappings fills it.

The arrival counters and the epoch are 32-bit words that wrap in a long-lived process; these
cases start them just below 2^31 so that exchanges cross the wrap, and check that a target
the pushes never reach makes the bounded wait give up: the device error word is set, the
output holds only the residual, and the context stays usable.  The layer itself is checked
against the oracle (dequantize-then-matmul in fp32, server/moe_layer_runtime.py:581-611) and
against the single-GPU fused layer.
"""
import time

import numpy as np
import pytest
import torch

from oracle import cases, router
from oracle.expert import DequantExpert
from oracle.layer import moe_layer

pytestmark = pytest.mark.gpu

E, H, I, G, TG, K = 16, 256, 128, 4, 2, 4
T = 24  # one column chunk of 1024 and 6 pushing CTAs of 4 tokens per exchange
CTAS = 6
X_INTS = T * H // 2  # the gathered rows: T x H 2-byte elements
TAIL = T * H + X_INTS  # int32 offset of the counters in the exchange buffer
FLAGS, EPOCH, GFLAGS, GEPOCH = TAIL, TAIL + 32, TAIL + 8, TAIL + 34


def s32(u: int) -> int:
    u &= 0xFFFFFFFF
    return u - (1 << 32) if u >= 1 << 31 else u


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def layer(dev):
    from constellation_b200.context import ExpertContext, MoEConfig

    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                    num_experts_per_tok=K)
    x = cases.activations(401, T, H)
    w, b = cases.router(401, E, H, bias_std=0.05)
    experts = {e: cases.expert(40100 + e, H, I) for e in range(E)}
    sh = cases.expert(40199, H, I)
    res = cases.activations(402, T, H)
    ctx = ExpertContext(dev, cfg, n_slots=E + 1, max_tokens=T)
    for e in range(E):
        ctx.upload_bundle(e, e, experts[e])
    ctx.upload_bundle(E, -1, sh)
    ref = moe_layer(x, w, b, {e: DequantExpert(v) for e, v in experts.items()}, DequantExpert(sh), n_group=G,
                    topk_group=TG, top_k=K)
    xt = torch.from_numpy(x).to(dev, torch.bfloat16)
    wt, bt = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
    rt = torch.from_numpy(res).to(dev)
    return ctx, xt, wt, bt, rt, ref, res


def peer_set(buf: torch.Tensor):
    from constellation_b200._lib import CstPeerSet

    ps = CstPeerSet()
    ps.world, ps.rank, ps.tl, ps.tl_cap = 1, 0, T, T
    base = buf.data_ptr()
    ps.recv[0] = base
    ps.flags[0] = base + FLAGS * 4
    ps.epoch = base + EPOCH * 4
    ps.done = base + (EPOCH + 1) * 4
    ps.x_offset = T * H * 4
    ps.gather_epoch = base + GEPOCH * 4
    return ps


def exchange(ctx, xt, wt, bt, rt, ps):
    idx, wts = ctx.route(xt, wt, bt)
    ctx.moe_routed_push(xt, idx, wts, ps)
    return ctx.reduce_pushed(ps, residual=rt, out_dtype=torch.float32)


def test_push_reduce_matches_layer_across_counter_wrap(layer, dev):
    ctx, xt, wt, bt, rt, ref, res = layer
    buf = torch.zeros(TAIL + 64, dtype=torch.int32, device=dev)
    start = (1 << 31) - 2 * CTAS - 3  # the third exchange carries both words past 2^31
    buf[FLAGS] = s32(start)
    buf[EPOCH] = s32(start)
    ps = peer_set(buf)
    outs = [exchange(ctx, xt, wt, bt, rt, ps) for _ in range(5)]
    ctx.device_error()  # no wait gave up
    assert int(buf[FLAGS]) == s32(start + 5 * CTAS) and int(buf[EPOCH]) == s32(start + 5 * CTAS)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # the fused single-GPU layer adds the same rows in the same order
    fused = ctx.moe_layer(xt, wt, bt, out_dtype=torch.float32) + rt
    torch.testing.assert_close(outs[0], fused, rtol=1e-5, atol=1e-5)
    idx, _, logits, _ = ctx.route(xt, wt, bt, return_aux=True)
    c = router.compare_routes(idx.cpu().numpy(), ref.route.topk_weight, xt.float().cpu().numpy(), wt.cpu().numpy(),
                              bt.cpu().numpy(), dev_logits=logits.cpu().numpy(), n_group=G, topk_group=TG, top_k=K)
    assert c["unexplained"] == 0, c
    ok = np.all(idx.cpu().numpy() == ref.route.topk_idx, axis=1)
    got = outs[0].cpu().numpy() - res
    rel = np.abs(got - ref.out_f32).max(axis=1) / np.abs(ref.out_f32).max(axis=1)
    assert float(rel[ok].max()) < 2e-3


def test_reduce_wait_gives_up_when_a_target_is_never_reached(layer, dev):
    """Counter just below 2^31, target just past it: a plain signed comparison reads the
    wrapped (negative) target as reached and sums whatever the slots hold; the wrapped
    difference waits, gives up, and reports it."""
    from constellation_b200._lib import CstError

    ctx, xt, wt, bt, rt, ref, res = layer
    buf = torch.zeros(TAIL + 64, dtype=torch.int32, device=dev)
    buf[FLAGS] = s32((1 << 31) - 4 * CTAS)
    buf[EPOCH] = s32((1 << 31) - 2)  # after the push: counter 2^31 - 3 CTAS, target 2^31 + 4
    ps = peer_set(buf)
    idx, wts = ctx.route(xt, wt, bt)
    ctx.moe_routed_push(xt, idx, wts, ps)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    out = ctx.reduce_pushed(ps, residual=rt, out_dtype=torch.float32)
    torch.cuda.synchronize(dev)
    waited = time.perf_counter() - t0
    print(f"bounded wait gave up after {waited:.3f} s")
    with pytest.raises(CstError):
        ctx.device_error()
    assert torch.equal(out, rt)  # only the residual
    assert waited < 30.0
    # the error word was cleared and the context still runs a full exchange
    buf2 = torch.zeros(TAIL + 64, dtype=torch.int32, device=dev)
    good = exchange(ctx, xt, wt, bt, rt, peer_set(buf2))
    ctx.device_error()
    fused = ctx.moe_layer(xt, wt, bt, out_dtype=torch.float32) + rt
    torch.testing.assert_close(good, fused, rtol=1e-5, atol=1e-5)


def test_gather_rows_across_counter_wrap_and_timeout(layer, dev):
    """cst_gather_rows on one rank: the rows land in the gathered slots (the layer over them
    equals the layer over x), across the 32-bit wrap of its counters; a gather target that is
    never reached gives up, sets the error word and leaves the context usable."""
    from constellation_b200._lib import CstError

    ctx, xt, wt, bt, rt, ref, res = layer
    buf = torch.zeros(TAIL + 64, dtype=torch.int32, device=dev)
    start = (1 << 31) - 9  # 6 row blocks per exchange: the second one wraps
    buf[GFLAGS] = s32(start)
    buf[GEPOCH] = s32(start)
    ps = peer_set(buf)
    gathered = buf[T * H:TAIL].view(torch.bfloat16).view(T, H)
    for i in range(3):
        ctx.gather_rows(xt, ps)
        ctx.device_error()
        assert torch.equal(gathered, xt), i
    assert int(buf[GFLAGS]) == s32(start + 3 * 6) and int(buf[GEPOCH]) == s32(start + 3 * 6)
    out = exchange(ctx, gathered, wt, bt, rt, ps)
    fused = ctx.moe_layer(xt, wt, bt, out_dtype=torch.float32) + rt
    torch.testing.assert_close(out, fused, rtol=1e-5, atol=1e-5)
    # a target ahead of what arrives: the wait gives up
    buf[GEPOCH] = s32(int(buf[GEPOCH]) + 100)
    ctx.gather_rows(xt, ps)
    with pytest.raises(CstError):
        ctx.device_error()
    ctx.device_error()  # cleared


def test_push_skips_tokens_without_rows_here(dev):
    """With presence words, a rank pushes nothing for a token it has no row for (only a 0
    word) and the owner adds only the present slots: here only experts 0-3 are resident and
    there is no shared expert, so most tokens have no row; the exchange must still equal the
    fused single-GPU layer, and a token without rows gets exactly its residual."""
    from constellation_b200.context import ExpertContext, MoEConfig

    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                    num_experts_per_tok=K)
    x = cases.activations(411, T, H)
    w, b = cases.router(411, E, H, bias_std=0.05)
    res = cases.activations(412, T, H)
    ctx = ExpertContext(dev, cfg, n_slots=4, max_tokens=T)
    for e in range(4):
        ctx.upload_bundle(e, e, cases.expert(41100 + e, H, I))
    xt = torch.from_numpy(x).to(dev, torch.bfloat16)
    wt, bt = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
    rt = torch.from_numpy(res).to(dev)
    pres_off = (TAIL + 64) * 4
    buf = torch.zeros(TAIL + 64 + T, dtype=torch.int32, device=dev)
    buf[TAIL + 64:] = 7  # stale words from an earlier exchange
    buf[:T * H] = torch.full((T * H,), 1.0, device=dev).view(torch.int32)  # stale partials
    ps = peer_set(buf)
    ps.presence_offset = pres_off
    got = exchange(ctx, xt, wt, bt, rt, ps)
    ctx.device_error()
    idx, _ = ctx.route(xt, wt, bt)
    present = (idx < 4).any(dim=1)
    assert 0 < int(present.sum()) < T  # both kinds of token occur
    assert torch.equal(buf[TAIL + 64:].bool(), present)
    fused = ctx.moe_layer(xt, wt, bt, add_shared=False, out_dtype=torch.float32) + rt
    torch.testing.assert_close(got, fused, rtol=1e-5, atol=1e-5)
    assert torch.equal(got[~present], rt[~present])
