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
