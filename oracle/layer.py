"""One MoE layer, routed + shared, with fp32 accumulation (CPU oracle; test infrastructure only).

Restates the reference path for a batch of tokens:

* routing: ``route_token_real`` (``server/moe_layer_runtime.py:232-408``) via
  ``oracle.router.route_batched``;
* routed experts: ``run_one_expert_reference`` math (``:581-611``) per (token, expert);
* combine: ``combine_outputs_torch`` (``:148-167``) -- ``combined += w_k * y_k`` in fp32
  in route order;
* shared expert: ``run_shared_expert_block`` (``server/deepseek_full_model_executor.py:264-316``)
  on all tokens;
* ``ffn_total = shared + routed`` (``server/full_model_runtime.py:348``).

The reference rounds the routed sum to the runtime dtype before adding the shared
expert and ships expert outputs as fp16 over its socket; the acceptance criterion of
this build is an fp32 accumulation, so this oracle keeps every step in fp32 and
rounds once (bf16, round-to-nearest-even) at the end.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .codec import decode_bf16, encode_bf16_rne
from .expert import DequantExpert
from .router import RouteResult, route_batched


@dataclass
class LayerResult:
    out_f32: np.ndarray      # [T, H] fp32, routed + shared
    out_bf16: np.ndarray     # [T, H] uint16 bf16 bits of out_f32
    routed_f32: np.ndarray   # [T, H]
    shared_f32: np.ndarray | None
    route: RouteResult


def moe_layer(x: np.ndarray, gate_weight: np.ndarray, bias: np.ndarray, experts, shared=None, *,
              n_group: int, topk_group: int, top_k: int, norm_topk_prob: bool = True,
              routed_scaling_factor: float = 2.5, resident_mask=None) -> LayerResult:
    """``experts``: mapping / callable ``eid -> DequantExpert``; ``shared``: DequantExpert or None."""
    x = np.atleast_2d(np.asarray(x, dtype=np.float32))
    T, H = x.shape
    r = route_batched(x, gate_weight, bias, n_group=n_group, topk_group=topk_group, top_k=top_k,
                      norm_topk_prob=norm_topk_prob,
                      routed_scaling_factor=routed_scaling_factor, resident_mask=resident_mask)
    get = experts if callable(experts) else experts.__getitem__
    k = r.topk_idx.shape[1]
    y_tk = np.zeros((T, k, H), dtype=np.float32)
    for e in np.unique(r.topk_idx):
        tt, kk = np.nonzero(r.topk_idx == e)
        y_tk[tt, kk] = get(int(e)).forward(x[tt])
    routed = np.zeros((T, H), dtype=np.float32)
    for j in range(k):
        routed = (routed + r.topk_weight[:, j:j + 1] * y_tk[:, j]).astype(np.float32)
    shared_y = shared.forward(x) if shared is not None else None
    out = routed if shared_y is None else (routed + shared_y).astype(np.float32)
    return LayerResult(out_f32=out, out_bf16=encode_bf16_rne(out), routed_f32=routed,
                       shared_f32=shared_y, route=r)


def moe_layer_tokens(x: np.ndarray, gate_weight: np.ndarray, bias: np.ndarray, get_bundle, shared_bundle, tokens, *,
                     n_group: int, topk_group: int, top_k: int, norm_topk_prob: bool = True,
                     routed_scaling_factor: float = 2.5, workers: int = 8):
    """The layer of ``moe_layer`` for full-size weights, computed for a subset of tokens.

    Routing runs for every token (it is cheap); expert outputs only for ``tokens``, with
    each touched expert dequantized once, used for its rows and dropped, so host memory
    stays at ``workers`` dequantized experts.  ``get_bundle(eid)`` returns the expert's six
    upload tensors as numpy (``w_up``, ``s_up``, ``w_gate``, ``s_gate``, ``w_down``,
    ``s_down``, ``block``); ``shared_bundle`` likewise or None.  Same arithmetic and
    accumulation order as ``moe_layer``.  Returns ``(RouteResult, out_f32 [len(tokens), H])``.
    """
    from concurrent.futures import ThreadPoolExecutor

    x = np.atleast_2d(np.asarray(x, dtype=np.float32))
    tokens = np.asarray(tokens, dtype=np.int64)
    r = route_batched(x, gate_weight, bias, n_group=n_group, topk_group=topk_group, top_k=top_k,
                      norm_topk_prob=norm_topk_prob, routed_scaling_factor=routed_scaling_factor)
    sub_idx = r.topk_idx[tokens]
    k = sub_idx.shape[1]
    xs = x[tokens]
    y_tk = np.zeros((tokens.size, k, x.shape[1]), dtype=np.float32)

    def one(e):
        tt, kk = np.nonzero(sub_idx == e)
        y = DequantExpert(get_bundle(int(e))).forward(xs[tt])
        return tt, kk, y

    jobs = [int(e) for e in np.unique(sub_idx)]
    shared_y = None
    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        sh = pool.submit(lambda: DequantExpert(shared_bundle).forward(xs)) if shared_bundle is not None else None
        for tt, kk, y in pool.map(one, jobs):
            y_tk[tt, kk] = y
        if sh is not None:
            shared_y = sh.result()
    routed = np.zeros((tokens.size, x.shape[1]), dtype=np.float32)
    w = r.topk_weight[tokens]
    for j in range(k):
        routed = (routed + w[:, j:j + 1] * y_tk[:, j]).astype(np.float32)
    out = routed if shared_y is None else (routed + shared_y).astype(np.float32)
    return r, out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 value, as fp32."""
    return decode_bf16(encode_bf16_rne(x))


def rms_norm(x: np.ndarray, weight: np.ndarray | None = None, eps: float = 1e-6) -> np.ndarray:
    """``x * rsqrt(mean(x^2) + eps) * weight`` in fp32 (the sparse-layer ``rms_norm``)."""
    x = np.asarray(x, dtype=np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    y = (x / np.sqrt(ms + eps)).astype(np.float32)
    if weight is not None:
        y = (y * np.asarray(weight, dtype=np.float32)).astype(np.float32)
    return y


def moe_stack(h: np.ndarray, layers, *, n_group: int, topk_group: int, top_k: int, eps: float = 1e-6,
              routed_scaling_factor: float = 2.5) -> np.ndarray:
    """Stacked sparse layers without attention: per layer ``xn = bf16(rms_norm(h, w))``
    (the prenorm, ``server/full_model_runtime.py:271-276``) and ``h = bf16(h + routed +
    shared)`` (``:348-355``), every sum in fp32 and one bf16 rounding per tensor handed on.
    ``layers``: sequence of ``(gate_weight, bias, experts, shared, norm_weight)``."""
    h = bf16_round(np.atleast_2d(np.asarray(h, dtype=np.float32)))
    for gate_weight, bias, experts, shared, norm_weight in layers:
        xn = bf16_round(rms_norm(h, norm_weight, eps))
        r = moe_layer(xn, gate_weight, bias, experts, shared, n_group=n_group, topk_group=topk_group, top_k=top_k,
                      routed_scaling_factor=routed_scaling_factor)
        h = bf16_round((h + r.out_f32).astype(np.float32))
    return h


__all__ = ["LayerResult", "moe_layer", "moe_layer_tokens", "moe_stack", "bf16_round", "rms_norm", "DequantExpert"]
