"""Batched sigmoid group-limited top-k router (CPU oracle; test infrastructure only).

Restates ``route_token_real`` (``server/moe_layer_runtime.py:232-408``) for a batch of
tokens, step by step:

1. ``logits = gate_weight @ hidden`` in fp32 (``:322``).  Here the dot products are
   accumulated in float64 and rounded once to float32 (the correctly rounded fp32
   logit); the reference's BLAS order differs only in the last ulp.
2. ``scores_raw = sigmoid(logits)`` (``:323``), ``scores_for_choice_raw = scores_raw +
   e_score_correction_bias`` (``:325``), both fp32.
3. Resident mask: non-resident experts get ``-inf`` in the choice scores and ``0`` in
   the unbiased scores (``:327-341``).
4. Group score = sum of the top-2 choice scores of each of ``n_group`` groups
   (``:343-345``); the ``topk_group`` best groups are kept (``:347-361``).
5. Top-``k`` experts over the group-masked choice scores (``:363-371``), with
   ``k = min(top_k, #resident)`` (``:365``).
6. Weights = the **unbiased** sigmoid scores of those experts (``:373``), divided by
   ``sum + 1e-20`` when ``norm_topk_prob`` and ``k > 1`` (``:376-378``), times
   ``routed_scaling_factor`` (``:381``).

Tie rule.  The reference calls ``torch.topk(..., sorted=False)``, whose order and tie
behaviour are unspecified.  This oracle (and the CUDA kernel) order every selection
by (value descending, index ascending): equal values go to the lowest index, and the
returned top-k list is sorted that way.  ``canonicalize`` sorts a reference route
list the same way so the two can be compared element by element.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class RouteResult:
    topk_idx: np.ndarray          # [T, k] int64, sorted by (choice desc, idx asc)
    topk_weight: np.ndarray       # [T, k] float32 (normalised, scaled)
    logits: np.ndarray            # [T, E] float32
    scores_raw: np.ndarray        # [T, E] float32
    scores_for_choice: np.ndarray  # [T, E] float32 (resident-masked, biased)
    group_scores: np.ndarray      # [T, G] float32
    selected_group_idx: np.ndarray  # [T, topk_group] int64 (sorted by score desc, idx asc)
    topk_choice_vals: np.ndarray  # [T, k] float32
    margin: np.ndarray            # [T] float64: min gap at the two selection boundaries


def _order_desc(vals: np.ndarray) -> np.ndarray:
    """argsort rows by (value desc, index asc); -inf sorts last, index breaks ties."""
    T, n = vals.shape
    idx = np.broadcast_to(np.arange(n), (T, n))
    # lexsort: last key is primary.  Negate values so that larger comes first.
    return np.lexsort((idx, -vals.astype(np.float64)), axis=-1)


def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def route_batched(hidden: np.ndarray, gate_weight: np.ndarray, bias: np.ndarray, *,
                  n_group: int, topk_group: int, top_k: int, norm_topk_prob: bool = True,
                  routed_scaling_factor: float = 2.5, resident_mask: np.ndarray | None = None,
                  logits: np.ndarray | None = None) -> RouteResult:
    hidden = np.atleast_2d(np.asarray(hidden, dtype=np.float32))
    gate_weight = np.asarray(gate_weight, dtype=np.float32)
    bias = np.asarray(bias, dtype=np.float32)
    T, H = hidden.shape
    E = gate_weight.shape[0]
    if gate_weight.shape[1] != H:
        raise RuntimeError("gate_weight / hidden size mismatch")
    if E % n_group != 0:
        raise RuntimeError(f"num_experts={E} not divisible by n_group={n_group}")
    if topk_group <= 0 or topk_group > n_group:
        raise RuntimeError(f"invalid topk_group={topk_group} for n_group={n_group}")
    if top_k <= 0 or top_k > E:
        raise RuntimeError(f"invalid top_k={top_k} for num_experts={E}")
    epg = E // n_group

    if logits is None:
        logits = (hidden.astype(np.float64) @ gate_weight.astype(np.float64).T).astype(np.float32)
    scores_raw = sigmoid_f32(logits)
    sfc_raw = (scores_raw + bias[None, :]).astype(np.float32)
    if resident_mask is None:
        resident = np.ones(E, dtype=bool)
    else:
        resident = np.asarray(resident_mask, dtype=bool)
        if not resident.any():
            raise RuntimeError("resident_expert_ids produced an empty resident mask")
    sfc = np.where(resident[None, :], sfc_raw, np.float32(-np.inf)).astype(np.float32)
    scores = np.where(resident[None, :], scores_raw, np.float32(0.0)).astype(np.float32)

    grouped = sfc.reshape(T, n_group, epg)
    top2 = -np.sort(-grouped, axis=-1)[..., :2]
    group_scores = (top2[..., 0] + top2[..., 1]).astype(np.float32)
    gorder = _order_desc(group_scores)
    sel_groups = gorder[:, :topk_group]
    gmask = np.zeros((T, n_group), dtype=bool)
    np.put_along_axis(gmask, sel_groups, True, axis=-1)
    score_mask = np.repeat(gmask, epg, axis=1)
    masked = np.where(score_mask, sfc, np.float32(-np.inf)).astype(np.float32)

    k = min(top_k, int(resident.sum()))
    eorder = _order_desc(masked)
    topk_idx = eorder[:, :k]
    choice_vals = np.take_along_axis(masked, topk_idx, axis=-1)
    w = np.take_along_axis(scores, topk_idx, axis=-1).astype(np.float32)
    if norm_topk_prob and k > 1:
        denom = np.zeros(T, dtype=np.float32)
        for j in range(k):  # sequential fp32 sum
            denom = (denom + w[:, j]).astype(np.float32)
        denom = (denom + np.float32(1e-20)).astype(np.float32)
        w = (w / denom[:, None]).astype(np.float32)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)

    # Near-tie margin: gap between the last kept and first dropped candidate at both
    # selection steps (group top-k, expert top-k), relative to the value scale.
    def gap(sorted_vals: np.ndarray, kk: int) -> np.ndarray:
        if kk >= sorted_vals.shape[1]:
            return np.full(sorted_vals.shape[0], np.inf)
        a = sorted_vals[:, kk - 1].astype(np.float64)
        b = sorted_vals[:, kk].astype(np.float64)
        with np.errstate(invalid="ignore"):
            g = np.where(np.isinf(b) & (b < 0), np.inf, np.abs(a - b))
        return g

    gs_sorted = np.take_along_axis(group_scores, gorder, axis=-1)
    es_sorted = np.take_along_axis(masked, eorder, axis=-1)
    # Which of two equal in-group values is "top-2" never changes the group sum, so
    # only the two cross-candidate boundaries can flip a selection.
    margin = np.minimum(gap(gs_sorted, topk_group), gap(es_sorted, k))
    return RouteResult(topk_idx=topk_idx.astype(np.int64), topk_weight=w, logits=logits,
                       scores_raw=scores_raw, scores_for_choice=sfc, group_scores=group_scores,
                       selected_group_idx=sel_groups.astype(np.int64),
                       topk_choice_vals=choice_vals, margin=margin)


def canonicalize(routes, scores_for_choice: np.ndarray | None = None):
    """Sort a reference route list ``[(eid, w), ...]`` by (choice desc, eid asc).

    With ``scores_for_choice`` (the reference aux array) the order follows the biased
    choice values like the oracle's; without it, by expert id.
    """
    routes = [(int(e), float(w)) for e, w in routes]
    if scores_for_choice is None:
        return sorted(routes, key=lambda r: r[0])
    sfc = np.asarray(scores_for_choice, dtype=np.float64)
    return sorted(routes, key=lambda r: (-sfc[r[0]], r[0]))


def compare_routes(dev_idx, dev_w, hidden, gate_weight, bias, *, dev_logits=None, near_tie: float = 1e-5,
                   **route_kw) -> dict:
    """Device routes against this oracle on EVERY token.

    ``dev_idx`` / ``dev_w``: ``[T, k]`` as the device returned them (order: choice desc,
    index asc, like the oracle).  ``dev_logits``: the device's own ``[T, E]`` fp32 logits,
    used only to explain a disagreement.

    Returns a dict:

    * ``tokens``; ``near_ties``: tokens whose oracle selection margin is ``<= near_tie``;
    * ``mismatched``: tokens whose index row differs from the oracle's;
    * ``explained``: mismatched tokens that are near-ties AND whose device selection this
      oracle reproduces exactly when it is given the device's fp32 logits instead of its own
      (correctly rounded, fp64-accumulated) ones -- the two then differ only in the last
      ulp of a logit, not in the selection logic;
    * ``unexplained`` = mismatched - explained (what a test asserts to be 0);
    * ``weight_max_rel``: max relative weight difference over the matching tokens, and
      ``weights_close``: every such weight within rtol 2e-6 + atol 1e-7 (the tolerance the
      tests hold the device weights to);
    * ``max_logit_abs_diff`` (with ``dev_logits``): device vs correctly rounded logits.
    """
    dev_idx = np.asarray(dev_idx).astype(np.int64)
    dev_w = np.asarray(dev_w, dtype=np.float32)
    r = route_batched(hidden, gate_weight, bias, **route_kw)
    same = np.all(dev_idx == r.topk_idx, axis=1)
    mism = np.nonzero(~same)[0]
    near = r.margin <= near_tie
    explained = 0
    if mism.size and dev_logits is not None:
        dl = np.asarray(dev_logits, dtype=np.float32)
        r2 = route_batched(np.asarray(hidden)[mism], gate_weight, bias, logits=dl[mism], **route_kw)
        ok = np.all(r2.topk_idx == dev_idx[mism], axis=1) & near[mism]
        explained = int(ok.sum())
    wrel = 0.0
    close = True
    if same.any():
        a = dev_w[same].astype(np.float64)
        b = r.topk_weight[same].astype(np.float64)
        wrel = float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30)))
        close = bool(np.all(np.abs(a - b) <= 2e-6 * np.abs(b) + 1e-7))
    out = {"tokens": int(dev_idx.shape[0]), "near_ties": int(near.sum()), "mismatched": int(mism.size),
           "explained": explained, "unexplained": int(mism.size) - explained, "weight_max_rel": wrel,
           "weights_close": close,
           "mismatched_tokens": [int(t) for t in mism[:16]]}
    if dev_logits is not None:
        out["max_logit_abs_diff"] = float(np.max(np.abs(np.asarray(dev_logits, np.float64) - r.logits)))
    return out
