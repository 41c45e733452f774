"""The allocation-free router entry point (cst_route_noalloc) against cst_route.

Callers that cannot call cudaMalloc -- a host runtime whose pool already owns the device
memory, or a process that must not grow after start-up -- route through
cst_route_noalloc, whose scratch is a static device array in the library.  This test
calls it through the C ABI twice in a row on different inputs and checks each result
against the context-based cst_route with the routing tolerance of the other tests
(indices bit-exact, weights rtol 2e-6), and checks that an oversized call is refused
with a message naming the limit.  The file name sorts last so a run that stops at the
first failure has run every other test first; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, H, G, TG, K = 256, 7168, 8, 4, 8


def _noalloc(lib, x, w, b, T, idx, wt, stream):
    return lib.cst_route_noalloc(x.data_ptr(), 2, T, H, w.data_ptr(), b.data_ptr(), None, E, G, TG, K, 1,
                                 ctypes.c_float(2.5), idx.data_ptr(), wt.data_ptr(), stream)


def test_route_noalloc_matches_cst_route_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from constellation_b200 import _lib
    from constellation_b200.context import ExpertContext, MoEConfig
    from oracle import cases

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T = 64
    w_np, b_np = cases.router(91, E, H)
    w, b = torch.from_numpy(w_np).to(dev), torch.from_numpy(b_np).to(dev)
    ctx = ExpertContext(dev, MoEConfig(), n_slots=0, max_tokens=T)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, seed in enumerate((92, 93)):
        x = torch.from_numpy(cases.activations(seed, T, H)).to(dev, torch.bfloat16)
        ref_idx, ref_w = ctx.route(x, w, b)
        idx = torch.full((T, K), -1, dtype=torch.int32, device=dev)
        wt = torch.zeros((T, K), dtype=torch.float32, device=dev)
        rc = _noalloc(_lib.lib, x, w, b, T, idx, wt, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize(dev)
        assert torch.equal(idx, ref_idx), f"call {call}: indices differ"
        np.testing.assert_allclose(wt.cpu().numpy(), ref_w.cpu().numpy(), rtol=2e-6, atol=0)
    ctx.device_error()


def test_route_noalloc_rejects_sizes_beyond_its_static_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from constellation_b200 import _lib

    dev = torch.device("cuda", 0)
    T = 2049  # 2049 * 256 floats > 2 MiB
    x = torch.zeros((T, H), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((E, H), dtype=torch.float32, device=dev)
    b = torch.zeros(E, dtype=torch.float32, device=dev)
    idx = torch.empty((T, K), dtype=torch.int32, device=dev)
    wt = torch.empty((T, K), dtype=torch.float32, device=dev)
    rc = _noalloc(_lib.lib, x, w, b, T, idx, wt, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.CST_ERR_INVALID_ARG
    assert "T <= 2048" in _lib.last_error()


def test_route_noalloc_large_batch_on_cuda_cores_twice():
    """128 experts x 2100 tokens fits the static scratch; cst_route takes its tensor-core
    logits there while the allocation-free entry point stays on the CUDA-core kernel (no
    device waits, nothing to report a timeout into).  Both are checked against the CPU
    oracle on every token (equal up to explained last-ulp near-ties), and against each
    other on two calls in a row."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from constellation_b200 import _lib
    from constellation_b200.context import ExpertContext, MoEConfig
    from oracle import cases, router

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, E2, G2, TG2 = 2100, 128, 8, 4
    w_np, b_np = cases.router(94, E2, H)
    w, b = torch.from_numpy(w_np).to(dev), torch.from_numpy(b_np).to(dev)
    ctx = ExpertContext(dev, MoEConfig(n_routed_experts=E2, n_group=G2, topk_group=TG2), n_slots=0, max_tokens=T)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, seed in enumerate((95, 96)):
        x_np = cases.activations(seed, T, H)
        x = torch.from_numpy(x_np).to(dev, torch.bfloat16)
        ref_idx, ref_w = ctx.route(x, w, b)
        idx = torch.full((T, K), -1, dtype=torch.int32, device=dev)
        wt = torch.zeros((T, K), dtype=torch.float32, device=dev)
        rc = lib_noalloc(_lib.lib, x, w, b, T, idx, wt, stream, E2, G2, TG2)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize(dev)
        xf = x.float().cpu().numpy()
        kw = dict(n_group=G2, topk_group=TG2, top_k=K)
        c_na = router.compare_routes(idx.cpu().numpy(), wt.cpu().numpy(), xf, w_np, b_np, **kw)
        c_rt = router.compare_routes(ref_idx.cpu().numpy(), ref_w.cpu().numpy(), xf, w_np, b_np, **kw)
        # without device logits a disagreement cannot be explained: it may only be a near-tie
        near = router.route_batched(xf, w_np, b_np, **kw).margin <= 1e-5
        for c in (c_na, c_rt):
            assert all(near[t] for t in c["mismatched_tokens"]), c
            assert c["mismatched"] <= int(near.sum()), c
        same = (idx == ref_idx).all(dim=1)
        assert int((~same).sum()) <= int(near.sum()), f"call {call}"
        np.testing.assert_allclose(wt[same].cpu().numpy(), ref_w[same].cpu().numpy(), rtol=2e-6, atol=0)
    ctx.device_error()


def lib_noalloc(lib, x, w, b, T, idx, wt, stream, n_experts, n_group, topk_group):
    return lib.cst_route_noalloc(x.data_ptr(), 2, T, H, w.data_ptr(), b.data_ptr(), None, n_experts, n_group,
                                 topk_group, K, 1, ctypes.c_float(2.5), idx.data_ptr(), wt.data_ptr(), stream)
