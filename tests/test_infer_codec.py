"""The expert node's InferRequest / InferResponse bodies on the CPU: the oracle restatement
and the library's codec (``constellation_b200.protocol`` over ``cst_*_infer_*``) against
bodies made by the reference's own C++ codec (``common/infer_codec.cc``) and Python codec
(``common/protocol.py``) -- ``tests/golden/infer_codec_golden.npz`` -- plus the request
handler's answers that need no device (a body that does not decode, an unknown layer).
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest

from oracle import infer_codec as oracle_codec

GOLDEN = Path(__file__).resolve().parent / "golden" / "infer_codec_golden.npz"
REQ_KEYS = ("expert_id", "batch_size", "hidden_dim", "input_dtype", "output_dtype")
RESP_KEYS = ("status_code", "batch_size", "hidden_dim", "output_dtype")


def _split(g, name):
    data, off = g[name], g[name + "_off"]
    return [bytes(data[off[i]:off[i + 1]]) for i in range(len(off) - 1)]


@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    out = {}
    for kind, fixed in (("req", 24), ("resp", 20)):
        bodies = _split(g, f"{kind}_body")
        out[kind] = [(tuple(int(v) for v in f), b[fixed:], b) for f, b in zip(g[f"{kind}_fields"], bodies)]
        out[f"bad_{kind}"] = _split(g, f"bad_{kind}")
    return out


@pytest.mark.parametrize("kind", ["req", "resp"])
def test_oracle_codec_matches_reference_bodies(golden, kind):
    long_kind = "request" if kind == "req" else "response"
    for fields, payload, body in golden[kind]:
        assert oracle_codec.encode(long_kind, fields, payload) == body
        assert oracle_codec.decode(long_kind, body) == (fields, payload)
    for bad in golden[f"bad_{kind}"]:
        assert oracle_codec.decode(long_kind, bad) is None


def test_library_codec_matches_reference_bodies(golden):
    from constellation_b200 import protocol as P

    for fields, payload, body in golden["req"]:
        msg = dict(zip(REQ_KEYS, fields), activation=payload)
        assert P.encode_infer_request(msg) == body
        assert P.decode_infer_request(body) == msg
        assert P.decode_infer_request(bytearray(body)) == msg
    for fields, payload, body in golden["resp"]:
        msg = dict(zip(RESP_KEYS, fields), output=payload)
        assert P.encode_infer_response(msg) == body
        assert P.decode_infer_response(body) == msg
    for bad in golden["bad_req"]:
        with pytest.raises(P.ProtocolError):
            P.decode_infer_request(bad)
    for bad in golden["bad_resp"]:
        with pytest.raises(P.ProtocolError):
            P.decode_infer_response(bad)


def test_library_codec_argument_errors():
    """The reference's encode errors (common/protocol.py:143-153, :505-507)."""
    from constellation_b200 import _lib
    from constellation_b200 import protocol as P

    ok = dict(expert_id=1, batch_size=1, hidden_dim=2, input_dtype=2, output_dtype=2, activation=b"abcd")
    with pytest.raises(ValueError, match="bytes-like"):
        P.encode_infer_request({**ok, "activation": "abcd"})
    with pytest.raises(ValueError, match="i32 out of range"):
        P.encode_infer_request({**ok, "expert_id": 2 ** 31})
    with pytest.raises(ValueError, match="u32 out of range"):
        P.encode_infer_request({**ok, "input_dtype": -1})
    # the C ABI reports the size it needs when the buffer is short
    m = _lib.CstInferRequest(1, 1, 2, 2, 2, 4, ctypes.cast(ctypes.c_char_p(b"abcd"), ctypes.c_void_p).value)
    need = ctypes.c_int64(0)
    small = (ctypes.c_uint8 * 27)()
    assert _lib.lib.cst_encode_infer_request(ctypes.byref(m), small, 27, ctypes.byref(need)) == _lib.CST_ERR_INVALID_ARG
    assert need.value == 28


def test_handler_answers_without_a_device():
    """A body that does not decode gets no reply; an expert whose layer has no context here
    gets status 1 with the request's batch / hidden / output dtype and no output
    (worker.cc:92-97, :112-130).  Neither touches a GPU."""
    from constellation_b200 import protocol as P
    from constellation_b200.worker import handle_infer_request

    req = dict(expert_id=3 * 256 + 5, batch_size=2, hidden_dim=4, input_dtype=2, output_dtype=1,
               activation=bytes(16))
    body = P.encode_infer_request(req)
    assert handle_infer_request([], body[:-1]) is None
    assert handle_infer_request([], body + b"\x00") is None
    for layers, eid in (([], req["expert_id"]), ([None] * 4, req["expert_id"]), ([None], -7)):
        resp = P.decode_infer_response(handle_infer_request(layers, P.encode_infer_request({**req, "expert_id": eid})))
        assert resp == dict(status_code=1, batch_size=2, hidden_dim=4, output_dtype=1, output=b"")
