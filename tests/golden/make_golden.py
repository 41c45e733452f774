"""Generate the golden fixtures in this folder from the REFERENCE implementation itself.

Run in a checkout that has the reference tree (``CONSTELLATION_REFERENCE_ROOT``):

    python tests/golden/make_golden.py

It imports the reference's own Python functions (``server.moe_layer_runtime.
route_token_real``, ``combine_outputs_torch``, ``server.fp8_utils.
dequant_fp8_weight_blockwise``, ``common.protocol``'s infer codec) and calls the
reference's C++ code compiled from its sources (``oracle/_ref/libref_expert.so``:
``RunExpertReferenceV2``, ``FillDummyExpertBundleV2``, the activation codec, the FP8
LUT, the node's InferRequest / InferResponse codec).  Inputs come
from seeded, version-independent streams (``oracle.detrand``), so most fixtures
store the seed and the reference's outputs only.  The fixtures pin the CPU oracle
(``tests/test_oracle_golden.py``) and, through it, the CUDA path.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle import cases, refbuild  # noqa: E402
from oracle.codec import decode_bf16, encode_bf16_rne  # noqa: E402

OUT = Path(__file__).resolve().parent
FP16, BF16 = 1, 2


def _ref_modules():
    root = refbuild.reference_root()
    if root is None:
        raise SystemExit("reference tree not found; set CONSTELLATION_REFERENCE_ROOT")
    sys.path.insert(0, str(root))
    import torch
    from server.fp8_utils import dequant_fp8_weight_blockwise
    from server.moe_layer_runtime import combine_outputs_torch, route_token_real
    return torch, route_token_real, combine_outputs_torch, dequant_fp8_weight_blockwise


ROUTER_CASES = [
    # name, seed, T, E, H, n_group, topk_group, top_k, bias_std, resident (None | "stride3" | "few")
    ("full", 11, 16, 256, 7168, 8, 4, 8, 0.01, None),
    ("small", 12, 48, 64, 256, 8, 4, 8, 0.01, None),
    ("bias_heavy", 13, 32, 64, 256, 8, 4, 8, 1.0, None),
    ("restricted", 14, 32, 64, 256, 8, 4, 8, 0.01, "stride3"),
    ("few_resident", 15, 16, 64, 256, 8, 4, 8, 0.01, "few"),
    ("g4_k6", 16, 24, 128, 512, 4, 2, 6, 0.05, None),
]


def _resident(kind, E):
    if kind is None:
        return None
    if kind == "stride3":
        return [e for e in range(E) if e % 3 != 1]
    if kind == "few":
        # fewer residents than top_k, two per populated group: every group that can be
        # selected has a finite score, so no -inf tie (whose order torch.topk leaves
        # unspecified) reaches the result
        return [1, 5, 9, 12, 40, 41]
    raise ValueError(kind)


def make_router(torch, route_token_real):
    out = {}
    for name, seed, T, E, H, G, TG, K, bstd, res in ROUTER_CASES:
        x = cases.activations(seed, T, H)
        w, b = cases.router(seed, E, H, bias_std=bstd)
        resident = _resident(res, E)
        k_eff = K if resident is None else min(K, len(resident))
        idx = np.full((T, k_eff), -1, np.int64)
        wts = np.zeros((T, k_eff), np.float32)
        gsc = np.zeros((T, G), np.float32)
        logits = np.zeros((T, E), np.float32)
        for t in range(T):
            routes, aux = route_token_real(
                torch.from_numpy(x[t].copy()), torch.from_numpy(w), torch.from_numpy(b),
                n_group=G, topk_group=TG, top_k=k_eff, norm_topk_prob=True,
                routed_scaling_factor=2.5, scoring_func="sigmoid", topk_method="noaux_tc",
                n_routed_experts=E, hidden_size=H, resident_expert_ids=resident, return_aux=True)
            sfc = aux["scores_for_choice"]
            order = sorted(range(len(routes)), key=lambda i: (-float(sfc[routes[i][0]]), routes[i][0]))
            idx[t] = [routes[i][0] for i in order]
            wts[t] = [routes[i][1] for i in order]
            gsc[t] = aux["group_scores"]
            logits[t] = aux["logits"]
        p = f"{name}__"
        out.update({p + "cfg": np.array([seed, T, E, H, G, TG, K], np.int64),
                    p + "bias_std": np.float32(bstd),
                    p + "resident": np.array(resident if resident is not None else [], np.int64),
                    p + "has_resident": np.int64(resident is not None),
                    p + "topk_idx": idx, p + "topk_weight": wts, p + "group_scores": gsc,
                    p + "logits": logits,
                    p + "x_checksum": np.float64(np.sum(x.astype(np.float64))),
                    p + "w_checksum": np.float64(np.sum(w.astype(np.float64)))})
    np.savez_compressed(OUT / "router_golden.npz", **out)


DEQUANT_CASES = [("sq", 21, 128, 256, 128), ("ragged", 22, 150, 170, 128), ("blk64", 23, 130, 70, 64)]


def make_dequant(torch, dequant):
    out = {}
    for name, seed, r, c, blk in DEQUANT_CASES:
        w = cases.random_fp8_bytes(seed, (r, c))
        s = np.abs(cases.detrand.normal(seed + 100, ((r + blk - 1) // blk, (c + blk - 1) // blk),
                                        std=0.01)).astype(np.float32) + np.float32(1e-4)
        wt = torch.from_numpy(w).view(torch.float8_e4m3fn)
        ref = dequant(wt, torch.from_numpy(s), block_size=blk).numpy()
        out.update({f"{name}__w": w, f"{name}__s": s, f"{name}__block": np.int64(blk),
                    f"{name}__out": ref})
    np.savez_compressed(OUT / "dequant_golden.npz", **out)


def make_expert():
    out = {}
    lib = refbuild.ref_lib()
    # the reference's dummy bundle at two shapes, every in/out dtype pair
    for name, H, I in [("dummy_small", 256, 128), ("dummy_full", 7168, 2048)]:
        e = refbuild.dummy_expert(H, I)
        xf = np.empty(H, np.float32)
        for din in (FP16, BF16):
            xb = np.empty(H, np.uint16)
            lib.ref_dummy_input(H, din, xf.ctypes.data_as(refbuild._f32p),
                                xb.ctypes.data_as(refbuild._u16p))
            for dout in (FP16, BF16):
                if name == "dummy_full" and (din, dout) not in ((FP16, FP16), (BF16, BF16)):
                    continue
                y, h = refbuild.ref_expert_reference(e, xb, din, dout)
                out[f"{name}__in{din}_out{dout}__x"] = xb
                out[f"{name}__in{din}_out{dout}__y"] = y[0]
                out[f"{name}__in{din}_out{dout}__h"] = h[0]
    # a seeded quantized expert with a batch of bf16 activations
    for name, seed, H, I, T in [("synth_small", 31, 256, 128, 6), ("synth_mid", 32, 1024, 512, 3)]:
        e = cases.expert(seed, H, I)
        x = cases.activations(seed + 1, T, H)
        xb = encode_bf16_rne(x)
        y, h = refbuild.ref_expert_reference(e, xb, BF16, BF16)
        out[f"{name}__cfg"] = np.array([seed, H, I, T], np.int64)
        out[f"{name}__y"] = y
        out[f"{name}__h"] = h
        out[f"{name}__wsum"] = np.array([int(e.w_up.sum()), int(e.w_gate.sum()), int(e.w_down.sum())],
                                        np.int64)
    np.savez_compressed(OUT / "expert_golden.npz", **out)


def make_codec_lut():
    lib = refbuild.ref_lib()
    vals = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 0.5, 0.25, 0.499914, 65504.0, 1e-3, -1e-3, 1e-4, -1e-4,
                  1e10, -1e10, 3.14159, 6.1e-5, 5.96e-8, 2.0 ** -24, 70000.0], np.float32),
        cases.detrand.normal(41, (2000,), std=3.0),
        (cases.detrand.normal(42, (500,), std=1.0) * np.float32(1e-5)).astype(np.float32),
    ]).astype(np.float32)
    bf16 = np.array([lib.ref_encode_bf16(float(v)) for v in vals], np.uint16)
    fp16 = np.array([lib.ref_encode_fp16(float(v)) for v in vals], np.uint16)
    bits = np.arange(0, 65536, 97, dtype=np.uint16)
    dbf = np.array([lib.ref_decode_bf16(int(b)) for b in bits], np.float32)
    dfp = np.array([lib.ref_decode_fp16(int(b)) for b in bits], np.float32)
    lut = {f"fmt{f}": np.array([lib.ref_decode_fp8(f, b) for b in range(256)], np.float32)
           for f in (0, 1, 2)}
    np.savez_compressed(OUT / "codec_golden.npz", vals=vals, enc_bf16=bf16, enc_fp16=fp16,
                        bits=bits, dec_bf16=dbf, dec_fp16=dfp, **lut)


LAYER_CASE = dict(seed=51, T=8, E=16, H=256, I=128, G=4, TG=2, K=4)


def make_layer(torch, route_token_real, combine_outputs_torch, dequant):
    c = LAYER_CASE
    x = cases.activations(c["seed"], c["T"], c["H"])
    w, b = cases.router(c["seed"], c["E"], c["H"], bias_std=0.05)

    def deq(e):
        f = lambda q, s: dequant(torch.from_numpy(q).view(torch.float8_e4m3fn), torch.from_numpy(s))  # noqa: E731
        return f(e.w_up, e.s_up), f(e.w_gate, e.s_gate), f(e.w_down, e.s_down)

    def run_expert(ws, xt):  # server/moe_layer_runtime.py:604-609
        up = torch.matmul(xt, ws[0].t())
        gate = torch.matmul(xt, ws[1].t())
        return torch.matmul(up * torch.nn.functional.silu(gate), ws[2].t())

    experts = {e: deq(cases.expert(1000 + e, c["H"], c["I"])) for e in range(c["E"])}
    shared = deq(cases.expert(999, c["H"], c["I"]))
    out = np.zeros((c["T"], c["H"]), np.float32)
    idx = np.zeros((c["T"], c["K"]), np.int64)
    for t in range(c["T"]):
        xt = torch.from_numpy(x[t].copy())
        routes, aux = route_token_real(
            xt, torch.from_numpy(w), torch.from_numpy(b), n_group=c["G"], topk_group=c["TG"],
            top_k=c["K"], norm_topk_prob=True, routed_scaling_factor=2.5, scoring_func="sigmoid",
            topk_method="noaux_tc", n_routed_experts=c["E"], hidden_size=c["H"], return_aux=True)
        sfc = aux["scores_for_choice"]
        idx[t] = sorted([r[0] for r in routes], key=lambda e: (-float(sfc[e]), e))
        weighted = [(e, wt, run_expert(experts[e], xt).numpy()) for e, wt in routes]
        routed = combine_outputs_torch(weighted, out_dtype=torch.float32).numpy()
        out[t] = routed + run_expert(shared, xt).numpy()
    np.savez_compressed(OUT / "layer_golden.npz", cfg=np.array(list(c.values()), np.int64),
                        out_f32=out, out_bf16=encode_bf16_rne(out), topk_idx=idx,
                        x_checksum=np.float64(np.sum(x.astype(np.float64))))
    assert np.all(np.isfinite(decode_bf16(encode_bf16_rne(out))))


INFER_REQUESTS = [
    # expert_id, batch_size, hidden_dim, input_dtype, output_dtype, payload bytes
    (0, 1, 7168, 2, 2, 14336),                        # one DeepSeek-V3 token, bf16 -> bf16
    (255, 1, 256, 1, 2, 512),
    (61 * 256 + 17, 3, 64, 2, 1, 384),                # a global id (layer 61)
    (-1, 0, 0, 0, 0, 0),                              # empty activation
    (2 ** 31 - 1, -5, -(2 ** 31), 0xFFFFFFFF, 7, 3),  # field extremes
]
INFER_RESPONSES = [
    # status_code, batch_size, hidden_dim, output_dtype, payload bytes
    (0, 1, 7168, 2, 14336),
    (1, 1, 7168, 2, 0),
    (2, 4, 256, 1, 0),
    (4, 0, 0, 0, 0),
    (-3, 2 ** 31 - 1, -1, 0xFFFFFFFF, 5),
]


def _concat(chunks):
    off = np.zeros(len(chunks) + 1, np.int64)
    off[1:] = np.cumsum([len(c) for c in chunks])
    return np.frombuffer(b"".join(chunks), np.uint8).copy(), off


def _malformed(body: bytes, fixed: int):
    """Bodies both reference decoders reject: cut inside each part, a trailing byte, and a
    payload length that overruns or underruns the body."""
    bad = [body[:n] for n in (0, 3, 4, fixed - 1, fixed, len(body) - 1)] + [body + b"\x00"]
    n = int.from_bytes(body[fixed - 4:fixed], "little")
    for m in (0xFFFFFFFF, n + 1, n - 1):
        bad.append(body[:fixed - 4] + int(m).to_bytes(4, "little") + body[fixed:])
    return bad


def make_infer_codec():
    """InferRequest / InferResponse bodies from the reference's C++ codec (compiled into
    libref_expert.so) and its Python codec (common/protocol.py), which must agree.  Each
    body's payload is its tail after the fixed fields."""
    root = refbuild.reference_root()
    sys.path.insert(0, str(root))
    from common import protocol as P  # the reference coordinator's codec

    rng = np.random.default_rng(20240611)
    out = {}
    for kind, cases_, fixed in (("req", INFER_REQUESTS, 24), ("resp", INFER_RESPONSES, 20)):
        long_kind = "request" if kind == "req" else "response"
        enc = P.encode_infer_request if kind == "req" else P.encode_infer_response
        dec = P.decode_infer_request if kind == "req" else P.decode_infer_response
        keys = (("expert_id", "batch_size", "hidden_dim", "input_dtype", "output_dtype") if kind == "req" else
                ("status_code", "batch_size", "hidden_dim", "output_dtype"))
        pkey = "activation" if kind == "req" else "output"
        fields, payloads, bodies = [], [], []
        for c in cases_:
            f, n = c[:-1], c[-1]
            payload = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
            body_cpp = refbuild.ref_encode_infer(long_kind, f, payload)
            body_py = enc({**dict(zip(keys, f)), pkey: payload})
            assert body_cpp == body_py, (kind, f)
            d = dec(body_py)
            assert tuple(d[k] for k in keys) == tuple(f) and d[pkey] == payload
            assert refbuild.ref_decode_infer(long_kind, body_cpp) == (tuple(f), payload)
            fields.append(f)
            payloads.append(payload)
            bodies.append(body_cpp)
        bad = _malformed(next(b for b, q in zip(bodies, payloads) if 0 < len(q) <= 1024), fixed)
        for b in bad:
            assert refbuild.ref_decode_infer(long_kind, b) is None
            try:
                dec(b)
            except P.ProtocolError:
                pass
            else:
                raise AssertionError(f"reference Python decoder accepted a malformed {long_kind}")
        out[f"{kind}_fields"] = np.array(fields, np.int64)
        out[f"{kind}_body"], out[f"{kind}_body_off"] = _concat(bodies)
        out[f"bad_{kind}"], out[f"bad_{kind}_off"] = _concat(bad)
    np.savez_compressed(OUT / "infer_codec_golden.npz", **out)


def main():
    refbuild.build()
    torch, route, combine, dequant = _ref_modules()
    torch.set_num_threads(8)
    make_codec_lut()
    make_dequant(torch, dequant)
    make_router(torch, route)
    make_expert()
    make_layer(torch, route, combine, dequant)
    make_infer_codec()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
