"""The expert node's request path on one GPU: request body in, response body out
(``constellation_b200.worker.handle_infer_request`` over ``cst_serve_infer_request``),
against the same context's ``cst_expert_forward`` (bit-identical: the same kernels) and the
oracle (dequantize-then-matmul in fp32, server/moe_layer_runtime.py:581-611), with the
worker's status codes (expert_node_v2/worker.cc:112-130,
backend/cuda/backend_workspace_cuda_v2.cc:139-181) for every way a request can fail.
"""
import numpy as np
import pytest
import torch

from oracle import cases
from oracle.codec import decode_bf16, decode_fp16, encode_bf16_rne
from oracle.expert import DequantExpert

pytestmark = pytest.mark.gpu

E, H, I = 16, 256, 128
FP16, BF16 = 1, 2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def node(dev):
    """Two layers on this GPU: layer 0 holds local experts 0-7, layer 1 holds 3 and 9."""
    from constellation_b200.context import ExpertContext, MoEConfig

    cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=4, topk_group=2,
                    num_experts_per_tok=4)
    held = {0: list(range(8)), 1: [3, 9]}
    layers, experts = [], {}
    for layer, ids in held.items():
        ctx = ExpertContext(dev, cfg, n_slots=len(ids), max_tokens=8, max_rows=24)
        for slot, e in enumerate(ids):
            experts[(layer, e)] = cases.expert(5000 + 100 * layer + e, H, I)
            ctx.upload_bundle(slot, e, experts[(layer, e)])
        layers.append(ctx)
    return layers, experts


def request(eid, x_bits, in_dt, out_dt, batch=None, hidden=H, activation=None):
    from constellation_b200 import protocol as P

    batch = x_bits.shape[0] if batch is None else batch
    act = x_bits.astype("<u2").tobytes() if activation is None else activation
    return P.encode_infer_request(dict(expert_id=eid, batch_size=batch, hidden_dim=hidden, input_dtype=in_dt,
                                       output_dtype=out_dt, activation=act))


def serve(layers, body):
    from constellation_b200 import protocol as P
    from constellation_b200.worker import handle_infer_request

    return P.decode_infer_response(handle_infer_request(layers, body, experts_per_layer=E))


def encode_x(x, dt):
    return encode_bf16_rne(x) if dt == BF16 else x.astype(np.float16).view(np.uint16)


def decode_y(bits, dt):
    return decode_bf16(bits) if dt == BF16 else decode_fp16(bits)


@pytest.mark.parametrize("layer,e,batch,in_dt,out_dt", [(1, 9, 1, BF16, BF16), (0, 5, 5, FP16, BF16),
                                                        (1, 3, 3, BF16, FP16), (0, 0, 24, FP16, FP16)])
def test_served_output_equals_expert_forward_and_oracle(dev, node, layer, e, batch, in_dt, out_dt):
    layers, experts = node
    x = cases.activations(700 + 10 * layer + e + batch, batch, H)
    xb = encode_x(x, in_dt)
    resp = serve(layers, request(layer * E + e, xb, in_dt, out_dt))
    assert (resp["status_code"], resp["batch_size"], resp["hidden_dim"], resp["output_dtype"]) == \
        (0, batch, H, out_dt)
    y = np.frombuffer(resp["output"], dtype="<u2").reshape(batch, H)
    # the same context's expert request on device tensors gives the same bits
    tdt = {BF16: torch.bfloat16, FP16: torch.float16}
    xt = torch.from_numpy(xb.view(np.int16)).view(tdt[in_dt]).to(dev)
    yt = layers[layer].expert_forward(e, xt, out_dtype=tdt[out_dt])
    assert np.array_equal(yt.cpu().view(torch.int16).numpy().view(np.uint16), y)
    ref = DequantExpert(experts[(layer, e)]).forward(decode_y(xb, in_dt))
    rel = np.abs(decode_y(y, out_dt) - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert float(rel.max()) < 1e-2


def test_status_codes_of_failed_requests(node):
    layers, _ = node
    x = encode_x(cases.activations(790, 2, H), BF16)
    fails = {
        1: [request(2 * E + 1, x, BF16, BF16),          # no context for layer 2
            request(-3, x, BF16, BF16)],
        2: [request(0 * E + 12, x, BF16, BF16),         # layer 0 does not hold expert 12
            request(1 * E + 0, x, BF16, BF16)],
        4: [request(5, x, BF16, BF16, hidden=128),      # hidden_dim is not the context's
            request(5, x, BF16, BF16, batch=3),         # activation bytes != batch x hidden x 2
            request(5, x[:0], BF16, BF16, batch=0),     # batch 0
            request(5, x, 3, BF16),                     # fp32 is not a wire dtype
            request(5, x, BF16, 0),
            request(5, np.zeros((25, H), np.uint16), BF16, BF16)],  # more rows than the context holds
    }
    from constellation_b200 import protocol as P

    for status, bodies in fails.items():
        for body in bodies:
            req = P.decode_infer_request(body)
            resp = serve(layers, body)
            assert resp == dict(status_code=status, batch_size=req["batch_size"], hidden_dim=req["hidden_dim"],
                                output_dtype=req["output_dtype"], output=b"")
    # the node still serves after every failure
    assert serve(layers, request(5, x, BF16, BF16))["status_code"] == 0
