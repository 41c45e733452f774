"""Expert parallelism for one MoE layer: one process per GPU, NCCL over NVLink/NVSwitch.

Replaces the reference's socket dispatch -- one TCP ``InferRequest`` per (token, expert),
run one after the other (``server/moe_layer_runtime.py:27-145``) -- with collectives
between the ranks of one node.  Expert ``e`` lives on rank ``e // experts_per_rank``
(contiguous blocks, the EP convention of the reference's patched HF model,
``tmp/patched_modeling/modeling_deepseek_eager.py:648-649``); tokens are sharded across
ranks; the router weights and the shared expert are replicated and every rank applies the
shared expert to its own tokens.

Three exchange strategies, all deterministic and all behind ``ExpertParallelMoE.forward``:

``allgather`` (default for decode)
    all-gather the tokens; every rank routes the whole gathered batch itself (the router is
    deterministic and its inputs are identical everywhere, so no routes are exchanged), runs
    its own experts on every row routed to them (routes to other ranks' experts are skipped
    by the packer) plus the shared expert on its own tokens in the same grouped launches,
    and reduce-scatters the fp32 partial sums back to the owning ranks.  Message sizes are
    fixed, so nothing waits on the host.  At decode batch the bytes match the all-to-all
    (T x H in, T x H x 4 back) because top_k equals the rank count at 8 GPUs.

``p2p``
    the all-gather exchange with the reduce-scatter fused into the combine: every rank
    stores each gathered token's partial sum straight into the owning rank's memory over
    NVLink (CUDA IPC mappings, ``constellation_b200.p2p``) and the owner adds the ranks'
    partials in rank order (``cst_moe_routed_push`` / ``cst_reduce_pushed``).

``alltoall`` (the NCCL all-to-all-v of the reference's expert-parallel model)
    exchange per-rank row counts (``all_to_all_single`` of ``world`` ints, the count step of
    ``modeling_deepseek_eager.py:656``), send each routed row to the rank that owns its
    expert (``:671-674``), run the grouped FFN on the received rows, send the weighted
    outputs back (``:780-790``) and combine at the source in fixed k order.  The split
    sizes must reach the host (NCCL takes host counts), which costs one device sync.

Hot-expert replicas (``all-gather`` and ``p2p`` modes).  With a skewed router (a prefill
chunk whose bias favours a few experts) the owners of the hot experts get most of the rows
and the step waits for them.  ``choose_replicas`` picks, from a calibration batch's routes,
the fewest hottest experts whose replication brings the busiest rank within ``target`` of
the mean; every rank then holds a copy of each and serves it for its OWN tokens only
(``ExpertContext.set_own_tokens_only``), while every other expert keeps its single owner.
Each (token, expert) row is still computed exactly once, by the same kernels, so the layer's
output is unchanged.

The communication plan (``plan_dispatch``) and the replica choice are plain torch / numpy
and run on any device, so the multi-rank host logic is tested on CPU with the gloo backend.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def rows_per_rank(topk_idx, world: int, n_experts: int, replicas=(), shared: bool = True) -> list[int]:
    """Packed rows each rank computes for a gathered batch ``topk_idx`` ([T, K], rank-major
    token shards): its own experts' routes from every token, the replicated experts' routes
    from its own tokens, plus one shared-expert row per own token."""
    import numpy as np

    idx = np.asarray(topk_idx)
    T = idx.shape[0]
    tl, epr = T // world, n_experts // world
    rep = np.zeros(n_experts, dtype=bool)
    rep[list(replicas)] = True
    owner = np.arange(n_experts) // epr
    out = []
    for r in range(world):
        own = (owner == r) & ~rep
        rows = int(own[idx].sum()) + int(rep[idx[r * tl:(r + 1) * tl]].sum())
        out.append(rows + (tl if shared else 0))
    return out


def choose_replicas(calib_topk_idx, world: int, n_experts: int, *, target: float = 1.1,
                    max_replicas: int = 32) -> list[int]:
    """The fewest hottest experts (by routes in the calibration batch) whose replication on
    every rank brings the busiest rank's rows within ``target`` x the mean (or the best of
    up to ``max_replicas``)."""
    import numpy as np

    idx = np.asarray(calib_topk_idx)
    if world <= 1:
        return []
    order = np.argsort(-np.bincount(idx.ravel(), minlength=n_experts), kind="stable")
    best, best_r = None, 0
    for r in range(0, max_replicas + 1):
        rows = rows_per_rank(idx, world, n_experts, order[:r].tolist())
        imb = max(rows) / (sum(rows) / len(rows))
        if best is None or imb < best - 1e-9:
            best, best_r = imb, r
        if imb <= target:
            return sorted(int(e) for e in order[:r])
    return sorted(int(e) for e in order[:best_r])


@dataclass
class DispatchPlan:
    order: torch.Tensor        # [Tl*K] flat (t, k) indices sorted by destination rank (stable)
    dest: torch.Tensor         # [Tl*K] destination rank of each flat route
    counts: torch.Tensor       # [world] rows sent to each rank
    inv: torch.Tensor          # [Tl, K] position of route (t, k) in the send order


def plan_dispatch(topk_idx: torch.Tensor, experts_per_rank: int, world: int) -> DispatchPlan:
    Tl, K = topk_idx.shape
    flat = topk_idx.reshape(-1).to(torch.int64)
    dest = torch.div(flat, experts_per_rank, rounding_mode="floor")
    order = torch.sort(dest * (Tl * K) + torch.arange(Tl * K, device=flat.device)).indices
    counts = torch.bincount(dest, minlength=world)[:world]
    inv = torch.empty_like(order)
    inv[order] = torch.arange(Tl * K, device=flat.device)
    return DispatchPlan(order=order, dest=dest, counts=counts, inv=inv.reshape(Tl, K))


class ExpertParallelMoE:
    """One MoE layer sharded over ``world`` ranks.

    ``compute`` is the rank's ``ExpertContext`` holding its ``experts_per_rank`` routed
    experts (router ids ``[rank * epr, (rank + 1) * epr)``) and the shared expert.
    """

    def __init__(self, compute, *, rank: int, world: int, n_routed_experts: int, group=None,
                 mode: str = "allgather", local_route_min: int = 128, p2p_tl_cap: int | None = None):
        if n_routed_experts % world:
            raise ValueError(f"{n_routed_experts} experts do not shard over {world} ranks")
        if mode not in ("allgather", "alltoall", "p2p"):
            raise ValueError(f"unknown EP mode {mode!r}")
        self.c = compute
        self.rank, self.world, self.group, self.mode = rank, world, group, mode
        self.E = n_routed_experts
        self.epr = n_routed_experts // world
        self._slot_map = None
        self._peers = None  # p2p mode: PeerExchange, created on the first forward
        #: p2p mode: tokens per rank the exchange buffers hold (default: the first forward's);
        #: a later forward with more tokens per rank raises
        self.p2p_tl_cap = None if p2p_tl_cap is None else int(p2p_tl_cap)
        #: all-gather mode: from this many tokens per rank on, each rank routes only its own
        #: tokens and the routes are gathered with the activations (a 2K-int row per token);
        #: below it every rank routes the whole gathered batch and no routes move
        self.local_route_min = int(local_route_min)
        #: set to a list to record (phase, CUDA event) pairs at the phase boundaries of forward()
        self.timeline: list | None = None

    def _mark(self, name: str) -> None:
        if self.timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.timeline.append((name, ev))

    # ------------------------------------------------------------------------------
    def slot_map(self, device) -> torch.Tensor:
        """Router expert id -> local arena slot (-1 elsewhere), on ``device``."""
        if self._slot_map is None:
            m = [self.c.find_slot(e) for e in range(self.E)]
            self._slot_map = torch.tensor(m, dtype=torch.int32, device=device)
        return self._slot_map

    def forward(self, x_local: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor, *,
                residual: torch.Tensor | None = None, resident: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        od = out_dtype or x_local.dtype
        Tl = x_local.shape[0]
        self._mark("start")
        if self.world == 1:
            topk_idx, topk_w = self.c.route(x_local, gate_weight, bias, resident=resident)
            self._mark("route")
            if residual is None:
                out = self.c.moe_routed_range(x_local, topk_idx, topk_w, 0, Tl, out_dtype=od)
            else:
                part = self.c.moe_routed_range(x_local, topk_idx, topk_w, 0, Tl, out_dtype=torch.float32)
                out = self.c.cast_extra(part, residual=residual, out_dtype=od)
            self._mark("experts")
            return out
        if self.mode == "allgather":
            return self._allgather(x_local, gate_weight, bias, resident, residual, od)
        if self.mode == "p2p":
            return self._p2p(x_local, gate_weight, bias, resident, residual, od)
        topk_idx, topk_w = self.c.route(x_local, gate_weight, bias, resident=resident)
        self._mark("route")
        return self._alltoall(x_local, topk_idx, topk_w, residual, od)

    def routes(self, x_all: torch.Tensor, gate_weight: torch.Tensor, bias: torch.Tensor, *,
               resident: torch.Tensor | None = None, return_logits: bool = False):
        """The routes ``forward`` computes for the gathered batch ``x_all`` (``[world * Tl, H]``,
        rank order): the same router calls over the same row sets -- the whole batch where
        every rank routes it, each rank's own rows where ranks route their own tokens -- so
        a checker can compare them with a reference without running the exchange."""
        Tl = x_all.shape[0] // self.world
        whole = self.world == 1 or self.mode == "p2p" or (self.mode == "allgather" and Tl < self.local_route_min)
        chunks = [x_all] if whole else [x_all[r * Tl:(r + 1) * Tl] for r in range(self.world)]
        parts = [self.c.route(ch, gate_weight, bias, resident=resident, return_aux=return_logits) for ch in chunks]
        idx = torch.cat([p[0] for p in parts])
        w = torch.cat([p[1] for p in parts])
        if return_logits:
            return idx, w, torch.cat([p[2] for p in parts])
        return idx, w

    # ------------------------------------------------------------------------------
    def _allgather(self, x_local, gate_weight, bias, resident, residual, od) -> torch.Tensor:
        Tl, H = x_local.shape
        x_all = torch.empty((self.world * Tl, H), dtype=x_local.dtype, device=x_local.device)
        if Tl >= self.local_route_min:
            # prefill-sized batches: route the own tokens, gather routes with the rows
            idx_l, w_l = self.c.route(x_local, gate_weight, bias, resident=resident)
            self._mark("route")
            K = idx_l.shape[1]
            meta = torch.cat([idx_l.to(torch.int32), w_l.view(torch.int32)], dim=1).contiguous()
            meta_all = torch.empty((self.world * Tl, 2 * K), dtype=torch.int32, device=x_local.device)
            dist.all_gather_into_tensor(x_all, x_local.contiguous(), group=self.group)
            dist.all_gather_into_tensor(meta_all, meta, group=self.group)
            idx_all = meta_all[:, :K].contiguous()
            w_all = meta_all[:, K:].contiguous().view(torch.float32)
            self._mark("all_gather")
        else:
            dist.all_gather_into_tensor(x_all, x_local.contiguous(), group=self.group)
            self._mark("all_gather")
            # Every rank routes the whole gathered batch itself: the router is deterministic
            # per token and its inputs are identical on all ranks, so all ranks agree on every
            # route without exchanging them.
            idx_all, w_all = self.c.route(x_all, gate_weight, bias, resident=resident)
            self._mark("route")
        # this rank's experts on every gathered row, the shared expert on its own tokens only
        lo = self.rank * Tl
        partial = self.c.moe_routed_range(x_all, idx_all, w_all, lo, lo + Tl, out_dtype=torch.float32)
        self._mark("experts")
        mine = torch.empty((Tl, H), dtype=torch.float32, device=x_local.device)
        dist.reduce_scatter_tensor(mine, partial, op=dist.ReduceOp.SUM, group=self.group)
        self._mark("reduce_scatter")
        out = self.c.cast_extra(mine, residual=residual, out_dtype=od)
        self._mark("cast")
        return out

    def _p2p(self, x_local, gate_weight, bias, resident, residual, od) -> torch.Tensor:
        """All-gather exchange over peer memory: every rank stores its rows into every rank's
        gathered rows (``cst_gather_rows``; NCCL all-gather for fp32 rows), and each gathered
        token's partial sum into the owning rank's memory, where the owner adds the ranks'
        partials (``cst_moe_routed_push`` / ``cst_reduce_pushed``).  A rank pushes the next
        call's rows only after its reduce of this call, which waited for every rank's push
        of this call's partials, so no slot is rewritten while its owner still reads it."""
        from .p2p import PeerExchange

        Tl, H = x_local.shape
        if Tl == 0:  # equal on every rank (the all-gather takes equal shares): nothing to exchange
            return torch.empty((0, H), dtype=od, device=x_local.device)
        if self._peers is None:
            self._peers = PeerExchange(x_local.device, world=self.world, rank=self.rank,
                                       tl_cap=max(Tl, self.p2p_tl_cap or 1), hidden=H, group=self.group)
        if Tl > self._peers.tl_cap:
            raise RuntimeError(f"p2p exchange was sized for {self._peers.tl_cap} tokens per rank, got {Tl}; "
                               "pass p2p_tl_cap= to size it for the largest batch")
        ps = self._peers.peer_set(Tl)
        if x_local.dtype in (torch.bfloat16, torch.float16):
            # the all-gather over peer memory: each rank stores its rows into every rank's
            # gathered rows and waits for the others' (cst_gather_rows)
            self.c.gather_rows(x_local.contiguous(), ps)
            x_all = self._peers.gathered(Tl, x_local.dtype)
        else:
            x_all = torch.empty((self.world * Tl, H), dtype=x_local.dtype, device=x_local.device)
            dist.all_gather_into_tensor(x_all, x_local.contiguous(), group=self.group)
        self._mark("all_gather")
        idx_all, w_all = self.c.route(x_all, gate_weight, bias, resident=resident)
        self._mark("route")
        self.c.moe_routed_push(x_all, idx_all, w_all, ps)
        self._mark("experts_push")
        out = self.c.reduce_pushed(ps, residual=residual, out_dtype=od)
        self._mark("reduce")
        return out

    def close(self) -> None:
        """Release the peer-exchange buffers (every rank, after its last forward)."""
        if self._peers is not None:
            torch.cuda.synchronize(self._peers.device)
            self._peers.close()
            self._peers = None

    def _alltoall(self, x_local, topk_idx, topk_w, residual, od) -> torch.Tensor:
        Tl, K = topk_idx.shape
        H = x_local.shape[1]
        dev = x_local.device
        plan = plan_dispatch(topk_idx, self.epr, self.world)
        counts_recv = torch.empty_like(plan.counts)
        dist.all_to_all_single(counts_recv, plan.counts, group=self.group)
        send_sizes = plan.counts.tolist()
        recv_sizes = counts_recv.tolist()
        n_recv = int(sum(recv_sizes))
        tok = torch.div(plan.order, K, rounding_mode="floor")
        x_send = x_local.index_select(0, tok)
        meta_send = torch.stack([topk_idx.reshape(-1)[plan.order].to(torch.int32),
                                 topk_w.reshape(-1)[plan.order].view(torch.int32)], dim=1).contiguous()
        x_recv = torch.empty((n_recv + Tl, H), dtype=x_local.dtype, device=dev)
        meta_recv = torch.empty((n_recv, 2), dtype=torch.int32, device=dev)
        dist.all_to_all_single(x_recv[:n_recv], x_send, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(meta_recv, meta_send, recv_sizes, send_sizes, group=self.group)
        # received routed rows + this rank's own tokens for the shared expert, one grouped call
        x_recv[n_recv:] = x_local
        shared_slot = self.c.find_shared_slot()
        slot = torch.cat([self.slot_map(dev)[meta_recv[:, 0].to(torch.int64)],
                          torch.full((Tl,), shared_slot, dtype=torch.int32, device=dev)])
        wts = torch.cat([meta_recv[:, 1].view(torch.float32), torch.ones(Tl, dtype=torch.float32, device=dev)])
        y_all = self.c.grouped_ffn(x_recv, slot, wts, out_dtype=torch.float32)
        rows = torch.empty((Tl * K + Tl, H), dtype=torch.float32, device=dev)
        dist.all_to_all_single(rows[:Tl * K], y_all[:n_recv], send_sizes, recv_sizes, group=self.group)
        rows[Tl * K:] = y_all[n_recv:]
        tk_row = torch.cat([plan.inv, torch.arange(Tl * K, Tl * K + Tl, device=dev)[:, None]], dim=1)
        return self.c.combine_rows(rows, tk_row, residual=residual, out_dtype=od)
