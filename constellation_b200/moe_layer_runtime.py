"""MoE-layer runtime with the interface of the reference's ``server/moe_layer_runtime.py``.

Same function names, arguments, return shapes and error classes as the reference, so a
caller of ``server.moe_layer_runtime`` switches by changing the import:

``route_token_real`` (``:232-408``), ``run_moe_layer`` (``:411-578``),
``run_topk_moe_layer`` (``:170-229``), ``dispatch_topk_experts`` (``:111-145``),
``infer_one_expert`` (``:27-81``), ``combine_outputs_torch`` (``:148-167``),
``validate_routes`` / ``normalize_routes`` (``:84-108``).

What changes underneath: there is no per-token Python loop and no socket.  Routing is the
fused CUDA router, dispatch is the device-side packer, the experts run as one grouped FP8
kernel per projection and the combine is one fp32 kernel -- all through the C ABI
(``include/constellation_b200.h``) on the layer's device.  The reference's entry points
take one token (1-D hidden); these accept 1-D (same results, routes in the canonical
order (biased score desc, expert id asc)) and also 2-D ``[T, hidden]`` batches.

``MoESession`` stands in for the reference's session object: the attributes these
functions read (``cfg``, ``get_router_config()``, ``backbone_store.layer(id)``,
``backbone_store.dtype``, ``coord.placements``) plus one ``ExpertContext`` per layer that
holds the layer's resident experts.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .expert_placement import (allowed_local_expert_ids_for_layer, make_global_expert_id,
                               split_global_expert_id)

FP16, BF16 = 1, 2  # common::ActivationDType


# ------------------------------------------------------------------------------------------
# session

@dataclass
class _Coord:
    placements: list = field(default_factory=list)


class _BackboneStore:
    def __init__(self, dtype: torch.dtype):
        self.dtype = dtype
        self._layers: dict[int, dict] = {}

    def layer(self, layer_id: int) -> dict:
        if int(layer_id) not in self._layers:
            raise KeyError(f"layer {layer_id} is not loaded")
        return self._layers[int(layer_id)]


class MoESession:
    """Holds what the runtime functions read from the reference's session."""

    def __init__(self, router_config: dict, *, experts_per_layer: int = 256, dtype=torch.bfloat16,
                 restricted_expert_ids=None, log_level: int = 0):
        self._router_config = dict(router_config)
        self.cfg = {"run": {"experts_per_layer": int(experts_per_layer),
                            "restricted_expert_ids": restricted_expert_ids},
                    "log_level": int(log_level)}
        self.backbone_store = _BackboneStore(dtype)
        self.coord = _Coord()
        self.contexts: dict[int, object] = {}

    def get_router_config(self) -> dict:
        return self._router_config

    def add_layer(self, layer_id: int, ctx, gate_weight: torch.Tensor, e_score_correction_bias: torch.Tensor,
                  *, host: str = "local", worker_port: int = 0, control_port: int = 0) -> None:
        """Register a layer: its ``ExpertContext`` (experts already uploaded) and router."""
        layer_id = int(layer_id)
        self.contexts[layer_id] = ctx
        self.backbone_store._layers[layer_id] = {
            "device": str(ctx.device),
            "router": {"gate_weight": gate_weight, "e_score_correction_bias": e_score_correction_bias},
        }
        epl = int(self.cfg["run"]["experts_per_layer"])
        for local in range(int(self._router_config["n_routed_experts"])):
            if ctx.find_slot(local) >= 0:
                self.coord.placements.append({
                    "expert_id": make_global_expert_id(layer_id, local, experts_per_layer=epl),
                    "host": host, "worker_port": worker_port, "control_port": control_port,
                })

    def context_for_global(self, expert_id: int):
        layer_id, local = split_global_expert_id(expert_id, int(self.cfg["run"]["experts_per_layer"]))
        ctx = self.contexts.get(layer_id)
        if ctx is None:
            raise RuntimeError(f"expert {expert_id} not found in placements")
        return ctx, local


# ------------------------------------------------------------------------------------------
# routing

_router_ctx: dict = {}


def _router_context(device: torch.device, *, E, H, n_group, topk_group, top_k, norm, scale, T):
    """A slot-less context (router workspace only), cached per shape and device."""
    from .context import ExpertContext, MoEConfig

    key = (str(device), E, H, n_group, topk_group, norm, float(scale))
    ctx = _router_ctx.get(key)
    if ctx is None or ctx.max_tokens < T or ctx.cfg.num_experts_per_tok < top_k:
        cfg = MoEConfig(hidden_size=H, moe_intermediate_size=128, n_routed_experts=E, n_group=n_group,
                        topk_group=topk_group, num_experts_per_tok=max(top_k, 1), norm_topk_prob=norm,
                        routed_scaling_factor=scale)
        ctx = ExpertContext(device, cfg, n_slots=0, max_tokens=max(T, 64))
        _router_ctx[key] = ctx
    return ctx


def _resident_mask(resident_expert_ids, E: int, device) -> tuple[torch.Tensor | None, int]:
    if resident_expert_ids is None:
        return None, E
    m = torch.zeros(E, dtype=torch.uint8)
    for eid in resident_expert_ids:
        eid = int(eid)
        if 0 <= eid < E:
            m[eid] = 1
    n = int(m.sum())
    if n == 0:
        raise RuntimeError("resident_expert_ids produced an empty resident mask")
    return m.to(device), n


def route_token_real(hidden, gate_weight: torch.Tensor, e_score_correction_bias: torch.Tensor, *, n_group: int,
                     topk_group: int, top_k: int, norm_topk_prob: bool, routed_scaling_factor: float,
                     scoring_func: str, topk_method: str, n_routed_experts: int, hidden_size: int,
                     resident_expert_ids=None, return_aux: bool = False):
    """Sigmoid group-limited top-k routing of one token (1-D) or a batch (2-D)."""
    if scoring_func != "sigmoid":
        raise RuntimeError(f"unsupported scoring_func={scoring_func}")
    if topk_method != "noaux_tc":
        raise RuntimeError(f"unsupported topk_method={topk_method}")
    for name, t in (("hidden", hidden), ("gate_weight", gate_weight),
                    ("e_score_correction_bias", e_score_correction_bias)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be torch.Tensor, got {type(t).__name__}")
    if hidden.ndim not in (1, 2):
        raise RuntimeError(f"hidden must be 1D (or 2D [T, H]), got shape={tuple(hidden.shape)}")
    if gate_weight.ndim != 2:
        raise RuntimeError(f"gate_weight must be 2D, got shape={tuple(gate_weight.shape)}")
    if e_score_correction_bias.ndim != 1:
        raise RuntimeError(f"e_score_correction_bias must be 1D, got shape={tuple(e_score_correction_bias.shape)}")
    dev = gate_weight.device
    if hidden.device != dev:
        raise RuntimeError(f"hidden device mismatch: hidden={hidden.device} gate_weight={gate_weight.device}")
    if e_score_correction_bias.device != dev:
        raise RuntimeError(f"bias device mismatch: bias={e_score_correction_bias.device} "
                           f"gate_weight={gate_weight.device}")
    if gate_weight.dtype != torch.float32:
        raise TypeError(f"gate_weight must be float32, got {gate_weight.dtype}")
    if e_score_correction_bias.dtype != torch.float32:
        raise TypeError(f"e_score_correction_bias must be float32, got {e_score_correction_bias.dtype}")
    if hidden.dtype != torch.float32:
        raise TypeError(f"hidden must be float32 for router scoring, got {hidden.dtype}. "
                        f"Cast it explicitly in the caller.")
    num_experts, gate_hidden = gate_weight.shape
    if topk_group <= 0 or topk_group > n_group:
        raise RuntimeError(f"invalid topk_group={topk_group} for n_group={n_group}")
    if top_k <= 0 or top_k > num_experts:
        raise RuntimeError(f"invalid top_k={top_k} for num_experts={num_experts}")
    if num_experts != n_routed_experts:
        raise RuntimeError(f"gate_weight shape {tuple(gate_weight.shape)} inconsistent with "
                           f"n_routed_experts={n_routed_experts}")
    if gate_hidden != hidden_size:
        raise RuntimeError(f"gate_weight shape {tuple(gate_weight.shape)} inconsistent with hidden_size={hidden_size}")
    if int(hidden.shape[-1]) != hidden_size:
        raise RuntimeError(f"hidden dim {int(hidden.shape[-1])} inconsistent with hidden_size={hidden_size}")
    if int(e_score_correction_bias.shape[0]) != num_experts:
        raise RuntimeError(f"bias shape {tuple(e_score_correction_bias.shape)} incompatible with "
                           f"num_experts={num_experts}")
    if num_experts % n_group != 0:
        raise RuntimeError(f"num_experts={num_experts} not divisible by n_group={n_group}")
    if dev.type != "cuda":
        raise RuntimeError("route_token_real runs on the CUDA router; move the router weights to a CUDA device")

    x2 = hidden.reshape(-1, hidden_size).contiguous()
    T = x2.shape[0]
    mask, n_res = _resident_mask(resident_expert_ids, num_experts, dev)
    k_eff = min(int(top_k), n_res)
    ctx = _router_context(dev, E=num_experts, H=hidden_size, n_group=n_group, topk_group=topk_group,
                          top_k=k_eff, norm=bool(norm_topk_prob), scale=float(routed_scaling_factor), T=T)
    idx, w, logits, gs = ctx.route(x2, gate_weight.contiguous(), e_score_correction_bias.contiguous(),
                                   resident=mask, top_k=k_eff, return_aux=True)
    idx_l = idx.tolist()
    w_l = w.tolist()
    routes_all = [[(int(e), float(v)) for e, v in zip(ri, rw)] for ri, rw in zip(idx_l, w_l)]
    routes = routes_all[0] if hidden.ndim == 1 else routes_all
    if not return_aux:
        return routes
    aux = _router_aux(logits, gs, idx, w, e_score_correction_bias, mask, n_group, topk_group, k_eff,
                      bool(norm_topk_prob), float(routed_scaling_factor), routes)
    if hidden.ndim == 1:
        aux = {k: (v[0] if isinstance(v, np.ndarray) and v.ndim >= 1 and k not in ("resident_mask",) else v)
               for k, v in aux.items()}
    return routes, aux


def _router_aux(logits, group_scores, idx, w, bias, mask, n_group, topk_group, k, norm, scale, routes):
    """The aux dict of route_token_real (``:389-407``) rebuilt from the kernel's logits."""
    E = logits.shape[1]
    scores_raw = torch.sigmoid(logits)
    sfc_raw = scores_raw + bias
    res = torch.ones(E, dtype=torch.bool, device=logits.device) if mask is None else mask.bool()
    sfc = sfc_raw.masked_fill(~res, float("-inf"))
    scores = scores_raw.masked_fill(~res, 0.0)
    order = torch.sort(group_scores, dim=-1, descending=True, stable=True).indices[:, :topk_group]
    gmask = torch.zeros_like(group_scores, dtype=torch.bool).scatter_(1, order, True)
    smask = gmask.repeat_interleave(E // n_group, dim=1)
    pre = scores.gather(1, idx.long())
    post = pre / (pre.sum(dim=1, keepdim=True) + 1e-20) if (norm and k > 1) else pre
    cv = sfc.masked_fill(~smask, float("-inf")).gather(1, idx.long())

    def n(t):
        return t.detach().cpu().numpy()

    return {"logits": n(logits), "scores_raw": n(scores_raw), "scores": n(scores),
            "scores_for_choice_raw": n(sfc_raw), "scores_for_choice": n(sfc), "group_scores": n(group_scores),
            "selected_group_idx": n(order), "group_mask": n(gmask), "score_mask": n(smask),
            "resident_mask": n(res), "topk_idx": n(idx.long()), "topk_choice_vals": n(cv),
            "topk_weight_pre_norm": n(pre), "topk_weight_post_norm": n(post), "topk_weight": n(w),
            "effective_top_k": int(k), "routes": routes}


# ------------------------------------------------------------------------------------------
# routes, dispatch, combine

def validate_routes(routes):
    if not routes:
        raise RuntimeError("routes is empty")
    seen = set()
    for expert_id, weight in routes:
        expert_id, weight = int(expert_id), float(weight)
        if expert_id in seen:
            raise RuntimeError(f"duplicate expert_id in routes: {expert_id}")
        seen.add(expert_id)
        if weight < 0:
            raise RuntimeError(f"negative route weight for expert {expert_id}: {weight}")


def normalize_routes(routes):
    validate_routes(routes)
    total = float(sum(float(w) for _, w in routes))
    if total == 0.0:
        raise RuntimeError("route weights sum to zero")
    return [(int(e), float(w) / total) for e, w in routes]


def combine_outputs_torch(weighted_outputs, *, out_dtype: torch.dtype, accum_dtype: torch.dtype = torch.float32,
                          device: str | torch.device = "cpu"):
    """``sum_k w_k * y_k`` in ``accum_dtype`` then cast (the per-route host combine)."""
    if not weighted_outputs:
        raise RuntimeError("weighted_outputs is empty")
    combined = None
    for _, weight, y in weighted_outputs:
        y_t = torch.as_tensor(y, dtype=accum_dtype, device=device)
        w_t = torch.as_tensor(weight, dtype=accum_dtype, device=device)
        combined = (w_t * y_t) if combined is None else combined.add_(w_t * y_t)
    return combined.to(dtype=out_dtype)


def infer_one_expert(session, expert_id: int, hidden: np.ndarray):
    """One global expert on one activation row, fp16 in / fp16 out like the reference's
    wire format (``:36-46``); returns ``{"output_dtype", "output", "array"}``."""
    ctx, local = session.context_for_global(int(expert_id))
    x = torch.as_tensor(np.asarray(hidden, dtype=np.float16).reshape(1, -1)).to(ctx.device)
    from ._lib import CstError

    try:
        y = ctx.expert_forward(local, x, out_dtype=torch.float16)
    except CstError as exc:
        raise RuntimeError(f"infer failed for expert {expert_id}: status={exc.code} output_dtype=None "
                           f"output_bytes=0") from exc
    arr = y.reshape(-1).cpu().numpy()
    return {"output_dtype": FP16, "output": arr.tobytes(), "array": arr}


def dispatch_topk_experts(session, hidden: np.ndarray, routes, *, return_aux: bool = False):
    """Per-route expert outputs, as the reference's sequential dispatch returns them."""
    validate_routes(routes)
    weighted_outputs = []
    expert_outputs = [] if return_aux else None
    for expert_id, weight in ((int(e), float(w)) for e, w in routes):
        resp = infer_one_expert(session, expert_id, hidden)
        y = np.asarray(resp["array"], dtype=np.float32)
        weighted_outputs.append((expert_id, weight, y))
        if return_aux:
            expert_outputs.append({"expert_id": expert_id, "weight": weight, "output": y.copy(),
                                   "weighted_output": (weight * y).astype(np.float32, copy=False),
                                   "output_dtype": int(resp["output_dtype"])})
    return (weighted_outputs, expert_outputs) if return_aux else weighted_outputs


def run_topk_moe_layer(session, hidden, routes, *, return_aux: bool = False,
                       accum_dtype: torch.dtype = torch.float32):
    """Routed experts for given global routes of ONE token + fp32 combine.

    Without ``return_aux`` this is one fused call on the device (grouped kernels +
    combine); ``weighted_outputs`` then lists ``(expert_id, weight, None)``.  With
    ``return_aux`` every expert's output is also materialised (per-route calls).
    """
    if not isinstance(hidden, torch.Tensor):
        raise TypeError(f"hidden must be torch.Tensor, got {type(hidden).__name__}")
    if hidden.ndim != 1:
        raise RuntimeError(f"hidden must be 1D, got shape={tuple(hidden.shape)}")
    validate_routes(routes)
    routes = [(int(e), float(w)) for e, w in routes]
    out_dtype = hidden.dtype
    if return_aux:
        h_np = hidden.detach().float().cpu().numpy()
        weighted, expert_outputs = dispatch_topk_experts(session, h_np, routes, return_aux=True)
        combined = combine_outputs_torch(weighted, out_dtype=out_dtype, accum_dtype=accum_dtype,
                                         device=hidden.device)
        return combined, weighted, expert_outputs
    ctx, _ = session.context_for_global(routes[0][0])
    locals_ = []
    for gid, w in routes:
        c2, loc = session.context_for_global(gid)
        if c2 is not ctx:
            raise RuntimeError("routes of one call must belong to one layer")
        locals_.append((loc, w))
    x = hidden.detach().to(ctx.device).reshape(1, -1)
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        x = x.float()
    idx = torch.tensor([[e for e, _ in locals_]], dtype=torch.int32, device=ctx.device)
    wt = torch.tensor([[w for _, w in locals_]], dtype=torch.float32, device=ctx.device)
    combined = ctx.moe_routed(x.contiguous(), idx, wt, add_shared=False, out_dtype=out_dtype).reshape(-1)
    return combined, [(gid, w, None) for gid, w in routes]


def _resident_local_ids(session, layer_id: int, router_cfg: dict) -> list[int]:
    restricted = session.cfg["run"].get("restricted_expert_ids")
    if restricted is not None:
        ids = sorted({int(x) for x in restricted})
        max_local = int(router_cfg["n_routed_experts"])
        for eid in ids:
            if eid < 0 or eid >= max_local:
                raise RuntimeError(f"restricted expert id out of range for layer {layer_id}: "
                                   f"{eid} not in [0, {max_local})")
        return ids
    return allowed_local_expert_ids_for_layer([int(p["expert_id"]) for p in session.coord.placements],
                                              layer_id=layer_id,
                                              experts_per_layer=int(session.cfg["run"]["experts_per_layer"]))


def run_moe_layer(session, hidden, layer_id: int, *, return_aux: bool = False):
    """Routed MoE output of one layer for one token (1-D) or a batch (2-D ``[T, H]``)."""
    layer_id = int(layer_id)
    if session.backbone_store is None:
        raise RuntimeError("session.backbone_store is not initialized")
    entry = session.backbone_store.layer(layer_id)
    dev = torch.device(entry["device"])
    runtime_dtype = session.backbone_store.dtype
    if not isinstance(hidden, torch.Tensor):
        raise TypeError(f"hidden must be torch.Tensor, got {type(hidden).__name__}")
    if hidden.ndim not in (1, 2):
        raise RuntimeError(f"hidden must be 1D (or 2D [T, H]), got shape={tuple(hidden.shape)}")
    rc = session.get_router_config()
    H = int(rc["hidden_size"])
    if int(hidden.shape[-1]) != H:
        raise RuntimeError(f"hidden size mismatch: got={int(hidden.shape[-1])} expected={H}")
    if "router" not in entry:
        raise RuntimeError(f"router weights are not loaded for layer {layer_id}")
    gw = entry["router"]["gate_weight"]
    bias = entry["router"]["e_score_correction_bias"]
    if not isinstance(gw, torch.Tensor):
        raise TypeError(f"gate_weight must be torch.Tensor, got {type(gw).__name__}")
    if not isinstance(bias, torch.Tensor):
        raise TypeError(f"e_score_correction_bias must be torch.Tensor, got {type(bias).__name__}")
    if gw.device != dev:
        raise RuntimeError(f"router gate_weight expected device={dev}, got device={gw.device}")
    if bias.device != dev:
        raise RuntimeError(f"router bias expected device={dev}, got device={bias.device}")
    if gw.dtype != torch.float32:
        raise TypeError(f"router gate_weight must be float32, got {gw.dtype}")
    if bias.dtype != torch.float32:
        raise TypeError(f"router e_score_correction_bias must be float32, got {bias.dtype}")
    resident = _resident_local_ids(session, layer_id, rc)
    if not resident:
        raise RuntimeError(f"no resident experts found for layer {layer_id}")
    ctx = session.contexts[layer_id]
    E = int(rc["n_routed_experts"])
    top_k = min(int(rc["top_k"]), len(resident))
    mask = torch.zeros(E, dtype=torch.uint8)
    mask[resident] = 1
    mask = mask.to(dev)
    x2 = hidden.detach().to(dev).reshape(-1, H).to(runtime_dtype).contiguous()
    epl = int(session.cfg["run"]["experts_per_layer"])
    if not return_aux:
        out = ctx.moe_layer(x2, gw, bias, resident=mask, top_k=top_k, add_shared=False, out_dtype=runtime_dtype)
        return {"output": out.reshape(hidden.shape)}
    out, idx, w = ctx.moe_layer(x2, gw, bias, resident=mask, top_k=top_k, add_shared=False,
                                out_dtype=runtime_dtype, return_routes=True)
    local_routes = [[(int(e), float(v)) for e, v in zip(ri, rw)] for ri, rw in zip(idx.tolist(), w.tolist())]
    global_routes = [[(make_global_expert_id(layer_id, e, experts_per_layer=epl), v) for e, v in r]
                     for r in local_routes]
    one = hidden.ndim == 1
    aux = {"layer_id": layer_id, "router_hidden": x2.float().cpu().numpy()[0 if one else slice(None)],
           "resident_local_expert_ids": resident,
           "routes": global_routes[0] if one else global_routes,
           "local_routes": local_routes[0] if one else local_routes,
           "selected_global_expert_ids": [[e for e, _ in r] for r in global_routes][0 if one else slice(None)],
           "selected_weights": [[v for _, v in r] for r in global_routes][0 if one else slice(None)],
           "topk_idx": idx.long().cpu().numpy()[0 if one else slice(None)],
           "topk_weight": w.cpu().numpy()[0 if one else slice(None)],
           "effective_top_k": top_k}
    if one:
        # the rest of the reference's aux for its 1-D call (:559-575): the router's own aux,
        # the per-route expert outputs (fp16 on the wire, as infer_one_expert returns them)
        # and their fp32 sum before the cast; "output" stays the fused result
        router_hidden = x2[0].float()
        _, raux = route_token_real(router_hidden, gw, bias, n_group=int(rc["n_group"]),
                                   topk_group=int(rc["topk_group"]), top_k=top_k,
                                   norm_topk_prob=bool(rc["norm_topk_prob"]),
                                   routed_scaling_factor=float(rc["routed_scaling_factor"]),
                                   scoring_func=str(rc.get("scoring_func", "sigmoid")),
                                   topk_method=str(rc.get("topk_method", "noaux_tc")), n_routed_experts=E,
                                   hidden_size=H, resident_expert_ids=resident, return_aux=True)
        combined, weighted, expert_outputs = run_topk_moe_layer(session, router_hidden, global_routes[0],
                                                                return_aux=True)
        aux = {"layer_id": layer_id, "router_hidden": aux["router_hidden"], **raux, **aux,
               "weighted_outputs": weighted, "combined_pre_cast": combined.detach().float().cpu().numpy(),
               "expert_outputs": expert_outputs}
    return {"output": out.reshape(hidden.shape), "aux": aux}


def run_sparse_moe_block(session, hidden: torch.Tensor, layer_id: int, *, residual: torch.Tensor | None = None):
    """Routed + shared expert (+ residual) of one layer in one fused call: the MoE part of
    ``run_sparse_layer`` (``server/full_model_runtime.py:283-355``) without its per-token loop."""
    entry = session.backbone_store.layer(int(layer_id))
    ctx = session.contexts[int(layer_id)]
    rc = session.get_router_config()
    x2 = hidden.reshape(-1, int(rc["hidden_size"])).to(session.backbone_store.dtype).contiguous()
    res2 = residual.reshape(x2.shape).to(x2.dtype).contiguous() if residual is not None else None
    out = ctx.moe_layer(x2, entry["router"]["gate_weight"], entry["router"]["e_score_correction_bias"],
                        add_shared=True, residual=res2)
    return out.reshape(hidden.shape)
