#!/usr/bin/env python
"""Benchmark of the B200 MoE-layer hot path (benchmark config 2, decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (``config.workload``): one DeepSeek-V3 MoE layer at decode batch T=64 (bf16
hidden 7168, 256 routed FP8 experts + 1 shared, n_group 8 / topk_group 4 / top_k 8,
scaling 2.5), experts sharded 256/N per GPU (expert parallel over NCCL for N > 1), tokens
sharded T/N per rank.  A step = one full layer: route -> dispatch -> grouped FP8 SwiGLU
-> combine + shared expert.  Total work is fixed as N grows ("scaling": "strong").  Weights
are seeded synthetic N(0, 0.02) quantized per 128x128 block (no checkpoint is available);
the 11.3 GB of expert weights (1.4 GB per GPU at N=8) exceed the 126 MB L2, so no flush is
needed between steps.

Printed (rank 0, one JSON line): tokens/s of the whole job (``value``), µs per layer, the
grouped-kernel roofline (algorithmic bytes / CUDA-event time vs the measured HBM copy
bandwidth), the same metric end to end through the public API with host buffers
(``e2e``), the reference CPU path timed on this host (``cpu_baseline``), and the SM clocks
sampled during the timed region.

``--impl reference`` times the reference's CPU implementation of the path on this host's
cores instead: the reference node's OpenMP FP8 expert kernels (compiled from the
reference sources into ``oracle/_ref``) at batch 1 per (token, expert), as the reference
runs them, plus the CPU restatement of its router and fp32 combine.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# Host thread pools, fixed before numpy or torch load: numpy's BLAS and torch's intra-op pool
# run one thread each, and only the reference's OpenMP expert kernels take the host cores
# (their thread count is an argument, ``host_cores()``).  Idle pools left spinning beside
# those kernels slowed them several times over; torchrun sets OMP_NUM_THREADS=1 for N > 1,
# so this also makes the CPU numbers the same at every N.
HOST_POOL_THREADS = 1
for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
    os.environ[_v] = str(HOST_POOL_THREADS)

H, I, E, G, TG, K = 7168, 2048, 256, 8, 4, 8
EXPERT_BYTES = 3 * I * H + 3 * (I // 128) * (H // 128) * 4  # 44,050,944
ROUTER_BYTES = E * H * 4 + E * 4
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--tokens", type=int, default=None,
                   help="tokens T of the whole job (default 64 for config2, 4096 for config4)")
    p.add_argument("--ep-mode", choices=["allgather", "alltoall", "p2p"], default="p2p",
                   help="expert-parallel exchange: NCCL all-gather + reduce-scatter, NCCL all-to-all-v, or "
                        "NCCL all-gather + the combine pushed to the token owners over peer memory")
    p.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying a CUDA graph")
    p.add_argument("--replicate-hot", default="auto",
                   help="expert parallelism: replicate the hottest experts on every rank, each rank serving "
                        "them for its own tokens ('auto': chosen from a calibration batch for config4 at N>1, "
                        "none otherwise; or a number of experts, 0 = none)")
    p.add_argument("--cpu-sample-tokens", type=int, default=2)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed layer's output")
    p.add_argument("--parity-tokens", type=int, default=4,
                   help="tokens whose layer output the CPU oracle recomputes (routes: every token)")
    p.add_argument("--layers", type=int, default=58, help="config3: stacked layers")
    p.add_argument("--workload", choices=["config2", "config1", "config3", "config4", "worker"], default="config2",
                   help="config2: the full decode layer, T=64 (default); config1: grouped FP8 expert matvec "
                        "only, 32 resident experts with n_e ~ U{1..16} rows each, 1 GPU; config4: one layer "
                        "over a 4096-token prefill chunk with a Zipf-skewed router bias; worker: the expert "
                        "node's InferRequest path, batch --tokens (default 1), 32 resident experts, 1 GPU")
    p.add_argument("--resident-experts", type=int, default=E,
                   help="upload only the first N routed experts of each rank (small profiling case; "
                        "routes to the others contribute nothing)")
    return p.parse_args()


def host_cores() -> int:
    """Host cores this process may run on (the affinity mask, not the machine's count)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def host_threads_note(cores: int) -> dict:
    return {"reference_kernels": cores, "omp_default": HOST_POOL_THREADS, "blas": HOST_POOL_THREADS}


def measured_peaks():
    f = REPO / "MEASURED_PEAKS.json"
    if f.is_file():
        try:
            d = json.loads(f.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def upgate_traffic(bytes_per_launch: int):
    """DRAM bytes of one decode up/gate launch: the traffic / algorithmic-bytes ratio that ncu
    measured on a scaled config-2 case (profiles/grouped_ffn_config2_dram_traffic.md: the
    weights stream once, so traffic grows with the experts a launch streams) times this
    launch's algorithmic bytes.  None when the summary is missing."""
    import re

    f = REPO / "profiles" / "grouped_ffn_config2_dram_traffic.md"
    try:
        m = re.search(r"traffic_per_algorithmic_byte_upgate:\s*([0-9.]+)", f.read_text())
    except OSError:
        return None
    if not m:
        return None
    return int(float(m.group(1)) * bytes_per_launch)


TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of a 54-expert config-2 up/gate launch "
                  "(traffic / algorithmic bytes = 1.0056), scaled by the experts this launch streams")


def fp8_peak_tflops():
    """Dense FP8 tensor peak: twice the measured bf16 GEMM rate (the FP8 rate itself is not
    in the measured file; B200's FP8 dense rate is twice its bf16 rate), else nominal."""
    f = REPO / "MEASURED_PEAKS.json"
    if f.is_file():
        try:
            d = json.loads(f.read_text())
            return 2.0 * float(d["bf16_tflops"]), "2 x measured bf16 (fp8 not measured)"
        except Exception:
            pass
    return 4500.0, "nominal fp8 dense"


def step_distribution(torch, run, k: int, dev, world: int = 1):
    """Per-step device times of ``k`` further steps -- CUDA events between consecutive steps
    on the launching stream, max over ranks per step -- as mean / p50 / p90 / p99 / max in
    ms (outside the timed region of the result line).  None if the events failed."""
    ms = [float("nan")] * k
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    try:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(k + 1)]
        torch.cuda.synchronize(dev)
        ev[0].record()
        for i in range(k):
            run()
            ev[i + 1].record()
        torch.cuda.synchronize(dev)
        ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(k)]
    except Exception:  # the distribution is informative only; every rank still joins the reduction
        pass
    t = torch.tensor(ms, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = sorted(float(v) for v in t.tolist())
    if not vals or any(v != v for v in vals):
        return None

    def pct(q):
        return round(vals[min(len(vals) - 1, int(round(q / 100 * (len(vals) - 1))))], 4)

    return {"n": k, "mean": round(sum(vals) / len(vals), 4), "p50": pct(50), "p90": pct(90), "p99": pct(99),
            "max": round(vals[-1], 4)}


def smi_gpu_id(torch, dev) -> str:
    """The device's PCI bus id in nvidia-smi's form.  nvidia-smi numbers GPUs in PCI order
    and ignores CUDA_VISIBLE_DEVICES, so a CUDA ordinal can name another GPU there."""
    p = torch.cuda.get_device_properties(dev)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of one GPU (``gpu``: PCI bus id), sampled every
    200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def _lines(self) -> int:
        self.f.flush()
        try:
            return sum(1 for line in Path(self.f.name).read_text().splitlines() if line.count(",") >= 8)
        except OSError:
            return 0

    def _wait_lines(self, n: int, limit_s: float) -> None:
        t_end = time.monotonic() + limit_s
        while self.p is not None and self._lines() < n and time.monotonic() < t_end and self.p.poll() is None:
            time.sleep(0.02)

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        # nvidia-smi can take longer than a short timed region to start on a busy box: wait
        # (bounded) for its first sample, so the region is bracketed by samples
        self._wait_lines(1, 5.0)
        self._n_enter = self._lines()
        return self

    def __exit__(self, *a):
        if self.p is not None:
            # one sample after the region started (the next 200 ms tick), then stop
            self._wait_lines(self._n_enter + 1, 1.0)
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(rows), "reasons": reasons, "gpu": self.gpu}


def rowwise_rel(a, ref) -> float:
    import numpy as np

    a = np.atleast_2d(a).astype(np.float64)
    ref = np.atleast_2d(ref).astype(np.float64)
    return float((np.abs(a - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)).max())


def layer_parity(torch, moe, rank, world, dev, x_all, gw, gb, out_local, n_tokens: int):
    """Correctness of the timed layer, checked outside the timed region at every N.

    The output rows of all ranks are gathered to rank 0 (NCCL, after timing).  Rank 0
    recomputes every token's routes with the router calls the layer made
    (``ExpertParallelMoE.routes``) and compares them with the CPU oracle of
    ``route_token_real`` on EVERY token; then the oracle recomputes the layer output
    (dequantize, then fp32 matmul, fp32 combine + shared) for ``n_tokens`` tokens spread over
    the batch -- so over the ranks -- regenerating only the experts those tokens reach from
    their seeds.  Returns the summary for the result line (rank 0) or None."""
    import torch.distributed as dist

    T = x_all.shape[0]
    if world > 1:
        out_all = torch.empty((T, H), dtype=out_local.dtype, device=dev)
        dist.all_gather_into_tensor(out_all, out_local.contiguous())
    else:
        out_all = out_local
    res = None
    if rank == 0:
        import numpy as np

        from constellation_b200 import synthetic
        from oracle import router as orouter
        from oracle.layer import moe_layer_tokens

        t0 = time.perf_counter()
        idx, w, logits = moe.routes(x_all, gw, gb, return_logits=True)
        torch.cuda.synchronize(dev)
        xh, gwh, gbh = x_all.float().cpu().numpy(), gw.cpu().numpy(), gb.cpu().numpy()
        kw = dict(n_group=G, topk_group=TG, top_k=K, norm_topk_prob=True, routed_scaling_factor=2.5)
        cmp = orouter.compare_routes(idx.cpu().numpy(), w.cpu().numpy(), xh, gwh, gbh,
                                     dev_logits=logits.cpu().numpy(), **kw)
        tokens = np.unique(np.linspace(0, T - 1, max(1, n_tokens)).round().astype(np.int64))

        def bundle(e):
            return synthetic.make_expert(H, I, seed=synthetic.expert_seed(e), device=dev).host()

        _, ref = moe_layer_tokens(xh, gwh, gbh, bundle, bundle(-1), tokens, workers=min(16, host_cores()), **kw)
        err = rowwise_rel(out_all.float().cpu().numpy()[tokens], ref)
        res = {"routes_checked_tokens": cmp["tokens"], "index_mismatch": cmp["mismatched"],
               "index_mismatch_unexplained": cmp["unexplained"], "near_ties": cmp["near_ties"],
               "weight_max_rel": cmp["weight_max_rel"], "output_checked_tokens": [int(t) for t in tokens],
               "output_max_rowwise_rel": err, "tol": 1e-2,
               "ok": bool(cmp["unexplained"] == 0 and err <= 1e-2),
               "oracle": "CPU restatement of route_token_real + dequantize-then-fp32-matmul experts + fp32 combine",
               "seconds": round(time.perf_counter() - t0, 1)}
    if world > 1:
        dist.barrier()
    return res


# ---------------------------------------------------------------------------------------
MAX_REPLICAS = 32


def setup_layer(torch, rank, world, T_total, dev, resident=E, zipf=False, spare_slots=0):
    from constellation_b200 import synthetic
    from constellation_b200.context import ExpertContext, MoEConfig

    cfg = MoEConfig()
    epr = E // world
    ctx = ExpertContext(dev, cfg, n_slots=epr + 1 + spare_slots, max_tokens=T_total)
    for j in range(min(epr, resident)):
        e = rank * epr + j
        ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(e), device=dev)
        ctx.upload_expert(j, e, ex.w_up, ex.s_up, ex.w_gate, ex.s_gate, ex.w_down, ex.s_down)
        del ex
    sh = synthetic.make_expert(H, I, seed=synthetic.expert_seed(-1), device=dev)
    ctx.upload_expert(epr, -1, sh.w_up, sh.s_up, sh.w_gate, sh.s_gate, sh.w_down, sh.s_down)
    del sh
    gw, gb = synthetic.make_router(H, E, seed=synthetic.router_seed(), device=dev)
    if zipf:  # config 4: router bias = 2.0 * log-Zipf(1.2) over a seeded permutation
        gb = synthetic.zipf_bias(E, seed=synthetic.router_seed(), device=dev)
    x_all = synthetic.make_activations(T_total, H, seed=synthetic.ACTIVATION_SEED, device=dev)
    Tl = T_total // world
    x = x_all[rank * Tl:(rank + 1) * Tl].contiguous()
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return ctx, gw, gb, x, x_all


def place_replicas(torch, ctx, rank, world, T, dev, gw, gb, how):
    """Hot-expert replicas for a skewed router: the experts to replicate come from a
    calibration batch (other activations than the timed ones, same router), chosen by
    ep.choose_replicas (or the N hottest for a number); each rank uploads the ones it does
    not own into spare slots and serves all of them for its own tokens only."""
    from constellation_b200 import ep, synthetic

    calib = synthetic.make_activations(T, H, seed=synthetic.ACTIVATION_SEED + 100, device=dev)
    idx, _ = ctx.route(calib, gw, gb)
    idx = idx.cpu().numpy()
    if how == "auto":
        reps = ep.choose_replicas(idx, world, E, max_replicas=MAX_REPLICAS)
    else:
        import numpy as np

        order = np.argsort(-np.bincount(idx.ravel(), minlength=E), kind="stable")
        reps = sorted(int(e) for e in order[:min(int(how), MAX_REPLICAS)])
    epr = E // world
    spare = epr + 1
    for e in reps:
        if not rank * epr <= e < (rank + 1) * epr:
            ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(e), device=dev)
            ctx.upload_expert(spare, e, ex.w_up, ex.s_up, ex.w_gate, ex.s_gate, ex.w_down, ex.s_down)
            spare += 1
            del ex
    for e in reps:
        ctx.set_own_tokens_only(e)
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return reps


def touched_experts(torch, ctx, gw, gb, x_all, resident=E):
    """Distinct routed experts the batch reaches among those with weights on the device."""
    idx, _ = ctx.route(x_all, gw, gb)
    u = torch.unique(idx)
    return int((u < resident).sum().item())


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
    prefill = args.workload == "config4"
    T = args.tokens or (4096 if prefill else 64)
    if T % world:
        raise SystemExit(f"T={T} does not shard over {world} ranks")
    from constellation_b200.ep import ExpertParallelMoE

    want_reps = world > 1 and args.ep_mode != "alltoall" and args.replicate_hot != "0" and \
        (args.replicate_hot != "auto" or prefill)
    ctx, gw, gb, x, x_all = setup_layer(torch, rank, world, T, dev, args.resident_experts, zipf=prefill,
                                        spare_slots=MAX_REPLICAS if want_reps else 0)
    replicas = place_replicas(torch, ctx, rank, world, T, dev, gw, gb, args.replicate_hot) if want_reps else []
    moe = ExpertParallelMoE(ctx, rank=rank, world=world, n_routed_experts=E, mode=args.ep_mode)
    out = torch.empty_like(x)

    def step():
        if world == 1:
            ctx.moe_layer(x, gw, gb, out=out)
        else:
            out.copy_(moe.forward(x, gw, gb))

    # the all-to-all-v exchange reads split sizes on the host, so it cannot be captured
    use_graph = (not args.no_graph) and (world == 1 or args.ep_mode in ("allgather", "p2p"))
    graph = None
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    if use_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
    # kernels of this library per layer (NCCL and torch copy kernels not counted)
    # (the packer is one launch up to 2048 routes and three beyond)
    launches_per_step = (8 if world == 1 else 9) + (2 if T * (K + 1) > 2048 else 0) + (1 if prefill else 0)

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    run = graph.replay if graph is not None else step
    with ClockSampler(smi_gpu_id(torch, dev)) as clk:
        ms_total = timed(run, args.steps)
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    value = T / (ms_step / 1e3)

    # end to end through the public API: pinned host input -> layer -> host output
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(out, device="cpu").pin_memory()

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        run()
        out_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps) / args.steps
    step_ms = step_distribution(torch, run, args.steps, dev, world)
    h2d = x_host.numel() * x_host.element_size() * world
    d2h = out_host.numel() * out_host.element_size() * world
    parity = None
    if not args.no_parity and args.resident_experts == E:
        run()
        torch.cuda.synchronize(dev)
        parity = layer_parity(torch, moe, rank, world, dev, x_all, gw, gb, out,
                              args.parity_tokens * (2 if prefill else 1))

    # per-stage device times (separate profiled pass) for the roofline
    ctx.profile(True)
    nprof = 10
    for _ in range(nprof):
        if world == 1:
            ctx.moe_layer(x, gw, gb, out=out)
        else:
            moe.forward(x, gw, gb)
    torch.cuda.synchronize(dev)
    stages = ctx.profile_read()
    ctx.profile(False)
    upg = [s["grouped_up_gate"] for s in stages if s["grouped_up_gate"] > 0]
    dn = [s["grouped_down"] for s in stages if s["grouped_down"] > 0]
    stage_ms = {k: statistics.mean(s[k] for s in stages) for k in stages[0]} if stages else {}
    # expert-parallel phases (gather / route / experts / reduce-scatter / cast), eager launches
    ep_phase_ms = None
    if world > 1:
        sums: dict = {}
        for _ in range(nprof):
            moe.timeline = []
            moe.forward(x, gw, gb)
            torch.cuda.synchronize(dev)
            tl = moe.timeline
            for (_, e0), (name, e1) in zip(tl[:-1], tl[1:]):
                sums[name] = sums.get(name, 0.0) + e0.elapsed_time(e1)
        moe.timeline = None
        ep_phase_ms = {k: round(v / nprof, 4) for k, v in sums.items()}

    # algorithmic bytes of the grouped kernels on this rank
    U_total = touched_experts(torch, ctx, gw, gb, x_all, args.resident_experts) if world == 1 else None
    if world > 1:
        idx, _ = ctx.route(x_all, gw, gb)
        lo, hi = rank * (E // world), (rank + 1) * (E // world)
        Tl = T // world
        rep_mask = torch.zeros(E, dtype=torch.bool, device=dev)
        rep_mask[list(replicas)] = True
        own = idx[(idx >= lo) & (idx < hi) & ~rep_mask[idx.long()]]
        mine = idx[rank * Tl:(rank + 1) * Tl]
        loc = torch.cat([own, mine[rep_mask[mine.long()]]])
        U_local = int(torch.unique(loc).numel())
        rows = int(loc.numel())
        U_t = torch.tensor([U_local], device=dev)
        dist.all_reduce(U_t)
        U_total = int(U_t.item())
    else:
        U_local = U_total
        rows = T * K
    rows_incl_shared = rows + T // world
    n_mat = U_local + 1
    grid = (I // 128) * (H // 128) * 4
    upg_bytes = n_mat * (2 * I * H + 2 * grid) + rows_incl_shared * (H * 2 + I * 4)
    dn_bytes = n_mat * (I * H + grid) + rows_incl_shared * (I * 4 + H * 4)
    peak, peak_kind = measured_peaks()
    upg_ms = statistics.mean(upg) if upg else float("nan")
    dn_ms = statistics.mean(dn) if dn else float("nan")
    ach_upg = upg_bytes / (upg_ms / 1e3) / 1e9
    pair_bytes = n_mat * EXPERT_BYTES + rows_incl_shared * (H * 2 + H * 4)
    ach_pair = pair_bytes / ((upg_ms + dn_ms) / 1e3) / 1e9
    layer_bytes = pair_bytes + ROUTER_BYTES + (T // world) * H * 4

    # config 4 is tensor-bound: natural FLOP (one product per weight element and row, the
    # activation terms not counted) against the FP8 dense peak
    flop_rank = rows_incl_shared * 3 * 2 * H * I
    flop_upg = rows_incl_shared * 2 * 2 * H * I
    fp8_peak, fp8_kind = fp8_peak_tflops()
    rows_t = torch.tensor([rows_incl_shared], device=dev, dtype=torch.float64)
    if world > 1:
        rows_all = [torch.zeros_like(rows_t) for _ in range(world)]
        dist.all_gather(rows_all, rows_t)
        rows_per_rank = [int(r.item()) for r in rows_all]
    else:
        rows_per_rank = [rows_incl_shared]
    imbalance = max(rows_per_rank) / (sum(rows_per_rank) / len(rows_per_rank))
    line = {
        "metric": "MoE-layer decode tokens/s (1 DeepSeek-V3 MoE layer, T=64, 256 FP8 experts + shared)",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "us_per_layer": round(ms_step * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3 weights x e4m3(3-term) activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, 128x128 block E4M3; RMS-normalised N(0,1) bf16 hidden)",
        "config": {"workload": "config2_decode_T64_one_layer", "tokens": T, "routed_experts": E,
                   "shared_expert": True, "hidden": H, "inter": I, "top_k": K,
                   "parallelism": f"ep{world}" + (f"_{args.ep_mode}" if world > 1 else ""),
                   "cuda_graph": graph is not None,
                   "touched_experts": U_total,
                   "l2": "no flush: 11.3 GB of expert weights (>= 1.2 GB per GPU) exceed the 126 MB L2"},
        "roofline": {"kernel": "grouped_ffn_tc up/gate (tcgen05 kind::f8f6f4, TMEM accumulators, TMA bulk ring)",
                     "bound": "hbm",
                     "achieved": round(ach_upg, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach_upg / peak, 4), "peak_source": peak_kind,
                     "bytes_per_launch": upg_bytes, "ms_per_launch": round(upg_ms, 4),
                     "traffic": upgate_traffic(upg_bytes), "traffic_source": TRAFFIC_SOURCE},
        "expert_matvec": {"kernels": "grouped up/gate + down", "bytes": pair_bytes,
                          "ms": round(upg_ms + dn_ms, 4), "achieved_gbs": round(ach_pair, 1),
                          "frac": round(ach_pair / peak, 4)},
        "layer_hbm": {"bytes_per_rank": layer_bytes, "achieved_gbs": round(layer_bytes / (ms_step / 1e3) / 1e9, 1),
                      "frac": round(layer_bytes / (ms_step / 1e3) / 1e9 / peak, 4)},
        "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "ep_phase_ms": ep_phase_ms,
        "step_ms": step_ms,
        "e2e": {"value": round(T / (ms_e2e / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms_e2e, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "parity": parity,
    }
    if prefill:
        tflops_upg = flop_upg / (upg_ms / 1e3) / 1e12
        tflops_layer = flop_rank / (ms_step / 1e3) / 1e12
        line["metric"] = f"MoE-layer prefill tokens/s (1 DeepSeek-V3 MoE layer, T={T}, Zipf-skewed routing)"
        line["dtype"] = "e4m3 weights x e4m3(2-term) activations, fp32 accumulate"
        line["config"]["workload"] = "config4_prefill_T4096_one_layer" if T == 4096 else f"config4_shape_T{T}"
        line["config"]["router_bias"] = "2.0 * log-Zipf(s=1.2) over a seeded permutation of the 256 experts"
        line["config"]["gemm_kernels"] = "prefill (128-row groups, 2 activation terms, one scale per row)"
        line["config"]["l2"] = ("no flush: 11.3 GB of expert weights (1.4 GB per GPU at N=8) and a "
                                f"{T * H * 2 / 1e6:.0f} MB activation batch exceed the 126 MB L2")
        line["roofline"] = {"kernel": "grouped_prefill up/gate (tcgen05 kind::f8f6f4, 128-row groups)",
                            "bound": "tensor", "achieved": round(tflops_upg, 1), "peak": round(fp8_peak, 1),
                            "unit": "TFLOP/s", "frac": round(tflops_upg / fp8_peak, 4), "peak_source": fp8_kind,
                            "flop_per_launch": flop_upg, "ms_per_launch": round(upg_ms, 4), "traffic": None}
        line["tensor_util"] = {"flop_per_rank": flop_rank, "layer_tflops_per_gpu": round(tflops_layer, 1),
                               "frac_of_fp8_peak": round(tflops_layer / fp8_peak, 4),
                               "flop_whole_job": int((K + 1) * T * 3 * 2 * H * I)}
        line["load_imbalance"] = {"rows_per_rank": rows_per_rank, "max_over_mean": round(imbalance, 3),
                                  "replicated_experts": replicas,
                                  "replica_choice": "ep.choose_replicas on a calibration batch (activation "
                                                    "seed + 100): fewest hottest experts with max/mean <= 1.1"
                                  if replicas else None}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_reference_rate(args.cpu_sample_tokens, args.cpu_seconds, T=T, zipf=prefill)
        except Exception as exc:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": f"{type(exc).__name__}: {exc}"}
    if graph is not None:
        torch.cuda.synchronize(dev)
        graph.reset()  # release the captured NCCL work before the process group goes away
        del graph
    if world > 1:
        dist.barrier()
        moe.close()  # every rank is done with the peer buffers
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


# ---------------------------------------------------------------------------------------
def run_config3(args):
    """Config 3: one decode step through ``--layers`` stacked MoE layers (58), T=128 tokens,
    experts sharded over the ranks; per layer prenorm -> MoE -> residual (MoEStack)."""
    import datetime

    import torch
    import torch.distributed as dist

    from constellation_b200 import synthetic
    from constellation_b200.context import ExpertContext, MoEConfig, rms_norm
    from constellation_b200.stack import MoEStack, StackLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, T = args.layers, args.tokens or 128
    epr = E // world
    need = L * (epr + 1) * EXPERT_BYTES
    if need > 0.85 * torch.cuda.get_device_properties(dev).total_memory:
        raise SystemExit(f"{L} layers need {need / 1e9:.0f} GB of expert weights per GPU at N={world}; "
                         "use more GPUs or --layers")
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=300))
    if T % world:
        raise SystemExit(f"T={T} does not shard over {world} ranks")
    Tl = T // world
    layers = []
    for l in range(L):
        ctx = ExpertContext(dev, MoEConfig(), n_slots=epr + 1, max_tokens=T)
        for j in range(epr):
            e = rank * epr + j
            ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(e, l), device=dev)
            ctx.upload_expert(j, e, ex.w_up, ex.s_up, ex.w_gate, ex.s_gate, ex.w_down, ex.s_down)
            del ex
        sh = synthetic.make_expert(H, I, seed=synthetic.expert_seed(-1, l), device=dev)
        ctx.upload_expert(epr, -1, sh.w_up, sh.s_up, sh.w_gate, sh.s_gate, sh.w_down, sh.s_down)
        del sh
        gw, gb = synthetic.make_router(H, E, seed=synthetic.router_seed(l), device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(synthetic.norm_seed(l))
        nw = (1.0 + 0.02 * torch.randn((H,), generator=g, device=dev)).contiguous()
        layers.append(StackLayer(ctx, gw, gb, nw))
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    stack = MoEStack(layers, rank=rank, world=world, n_routed_experts=E,
                     mode=args.ep_mode if args.ep_mode != "alltoall" else "allgather")
    h_all = synthetic.make_activations(T, H, seed=synthetic.ACTIVATION_SEED, device=dev)
    h0 = h_all[rank * Tl:(rank + 1) * Tl].contiguous()
    out = torch.empty_like(h0)

    def step():
        out.copy_(stack.forward(h0))

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    graph = None
    if not args.no_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
    run = graph.replay if graph is not None else step

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(smi_gpu_id(torch, dev)) as clk:
        ms_step = timed(run, args.steps) / args.steps
    clocks = clk.summary()
    h_host = h0.cpu().pin_memory()
    o_host = torch.empty_like(h_host).pin_memory()

    def e2e_step():
        h0.copy_(h_host, non_blocking=True)
        run()
        o_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps) / args.steps

    # algorithmic bytes on this rank: per layer its touched experts + shared + router, from
    # the routes each layer actually takes (one eager pass that also routes the gathered batch)
    touched = 0
    h = h0
    for layer, moe in zip(stack.layers, stack.moe):
        xn = rms_norm(h, layer.norm_weight, stack.eps)
        xa = torch.empty((T, H), dtype=xn.dtype, device=dev)
        if world > 1:
            dist.all_gather_into_tensor(xa, xn)
        else:
            xa.copy_(xn)
        idx, _ = layer.compute.route(xa, layer.gate_weight, layer.bias)
        lo, hi = rank * epr, (rank + 1) * epr
        touched += int(torch.unique(idx[(idx >= lo) & (idx < hi)]).numel())
        h = moe.forward(xn, layer.gate_weight, layer.bias, residual=h, out_dtype=h.dtype)
    bytes_rank = (touched + L) * EXPERT_BYTES + L * ROUTER_BYTES
    bt = torch.tensor([float(bytes_rank), float(touched)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(bt)
    peak, peak_kind = measured_peaks()
    ach = bytes_rank / (ms_step / 1e3) / 1e9
    line = {
        "metric": f"MoE decode step tokens/s ({L} stacked DeepSeek-V3 MoE layers, T={T})",
        "value": round(T / (ms_step / 1e3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "us_per_layer": round(ms_step * 1e3 / L, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3 weights x e4m3(3-term) activations, fp32 accumulate",
        "data": "synthetic (independently seeded N(0,0.02) weights per layer, 128x128 block E4M3; "
                "RMS-normalised N(0,1) bf16 hidden; prenorm weights 1 + N(0, 0.02))",
        "config": {"workload": "config3_decode_stack" if L == 58 else f"config3_shape_{L}_layers",
                   "layers": L, "tokens": T, "routed_experts": E, "shared_expert": True, "hidden": H, "inter": I,
                   "top_k": K, "parallelism": f"ep{world}" + (f"_{stack.moe[0].mode}" if world > 1 else ""),
                   "cuda_graph": graph is not None, "touched_experts_all_layers": int(bt[1].item()),
                   "l2": f"no flush: {L * (epr + 1) * EXPERT_BYTES / 1e9:.0f} GB of expert weights per GPU "
                         "exceed the 126 MB L2"},
        "roofline": {"kernel": "whole step (grouped tcgen05 expert kernels dominate)", "bound": "hbm",
                     "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                     "peak_source": peak_kind, "bytes_per_step_rank": bytes_rank, "traffic": None},
        "e2e": {"value": round(T / (ms_e2e / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms_e2e, 4),
                "h2d_bytes_per_step": h_host.numel() * 2 * world, "d2h_bytes_per_step": o_host.numel() * 2 * world},
        # per layer: rmsnorm, router 2, packer 1, pack x, up/gate, pack h, down, cast (+ NCCL)
        "gpu_launches": L * 10 * args.steps,
        "clocks": clocks,
    }
    if graph is not None:
        torch.cuda.synchronize(dev)
        graph.reset()
        del graph
    if world > 1:
        dist.barrier()
        stack.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


C1_EXPERTS = 32


def config1_rows(torch, seed=0):
    """Config 1's seeded batch: n_e ~ U{1..16} rows for each of the 32 experts, rows of
    one expert contiguous, bf16 N(0, 1) activations, routing weights U(0.05, 0.3)."""
    g = torch.Generator().manual_seed(seed)
    n_e = torch.randint(1, 17, (C1_EXPERTS,), generator=g)
    row_slot = torch.repeat_interleave(torch.arange(C1_EXPERTS, dtype=torch.int32), n_e)
    R = int(n_e.sum())
    x = torch.randn((R, H), generator=g).to(torch.bfloat16)
    w = 0.05 + 0.25 * torch.rand((R,), generator=g)
    return n_e, row_slot, x, w


def config1_bytes(R):
    """Algorithmic bytes of one config-1 call: every resident expert's weights and scales
    once, plus the bf16 rows read and the fp32 weighted rows written."""
    return C1_EXPERTS * EXPERT_BYTES + R * (H * 2 + H * 4)


def run_config1(args):
    import torch

    from constellation_b200 import synthetic
    from constellation_b200.context import ExpertContext, MoEConfig

    if int(os.environ.get("WORLD_SIZE", "1")) != 1 or args.gpus != 1:
        raise SystemExit("--workload config1 is a single-GPU configuration")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_e, row_slot_h, x_h, w_h = config1_rows(torch)
    R = x_h.shape[0]
    ctx = ExpertContext(dev, MoEConfig(), n_slots=C1_EXPERTS, max_tokens=64, max_rows=max(R, 64 * (K + 1)))
    for j in range(C1_EXPERTS):
        ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(j), device=dev)
        ctx.upload_expert(j, j, ex.w_up, ex.s_up, ex.w_gate, ex.s_gate, ex.w_down, ex.s_down)
        del ex
    x = x_h.to(dev)
    row_slot = row_slot_h.to(dev)
    rw = w_h.to(dev)
    y = torch.empty((R, H), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()

    def step():
        ctx.grouped_ffn(x, row_slot, rw, out=y)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    graph = None
    if not args.no_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
    run = graph.replay if graph is not None else step

    def timed(fn, k):
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b)

    with ClockSampler(smi_gpu_id(torch, dev)) as clk:
        ms_step = timed(run, args.steps) / args.steps
    clocks = clk.summary()
    nbytes = config1_bytes(R)
    value = nbytes / (ms_step / 1e3) / 1e9

    x_host = x_h.pin_memory()
    y_host = torch.empty((R, H), dtype=torch.float32).pin_memory()

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        run()
        y_host.copy_(y, non_blocking=True)

    for _ in range(3):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps) / args.steps
    step_ms = step_distribution(torch, run, args.steps, dev)

    ctx.profile(True)
    for _ in range(10):
        step()
    torch.cuda.synchronize(dev)
    stages = ctx.profile_read()
    ctx.profile(False)
    stage_ms = {k: statistics.mean(st[k] for st in stages) for k in stages[0]}
    upg_ms, dn_ms = stage_ms["grouped_up_gate"], stage_ms["grouped_down"]
    grid = (I // 128) * (H // 128) * 4
    upg_bytes = C1_EXPERTS * (2 * I * H + 2 * grid) + R * (H * 2 + I * 4)
    pair_bytes = nbytes
    peak, peak_kind = measured_peaks()
    ach_upg = upg_bytes / (upg_ms / 1e3) / 1e9
    ach_pair = pair_bytes / ((upg_ms + dn_ms) / 1e3) / 1e9
    line = {
        "metric": "expert-matvec HBM GB/s (grouped FP8 SwiGLU, 32 resident experts, n_e ~ U{1..16})",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 weights x e4m3(3-term) activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, 128x128 block E4M3; N(0,1) bf16 rows)",
        "config": {"workload": "config1_grouped_matvec_32experts", "experts": C1_EXPERTS, "rows": R,
                   "rows_per_expert": [int(v) for v in n_e], "hidden": H, "inter": I,
                   "bytes_per_step": nbytes, "cuda_graph": graph is not None,
                   "l2": "no flush: 1.41 GB of expert weights exceed the 126 MB L2"},
        "roofline": {"kernel": "grouped_ffn_tc up/gate (tcgen05 kind::f8f6f4, TMEM accumulators, TMA bulk ring)",
                     "bound": "hbm", "achieved": round(ach_upg, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach_upg / peak, 4), "peak_source": peak_kind,
                     "bytes_per_launch": upg_bytes, "ms_per_launch": round(upg_ms, 4),
                     "traffic": upgate_traffic(upg_bytes), "traffic_source": TRAFFIC_SOURCE},
        "expert_matvec": {"kernels": "grouped up/gate + down", "bytes": pair_bytes,
                          "ms": round(upg_ms + dn_ms, 4), "achieved_gbs": round(ach_pair, 1),
                          "frac": round(ach_pair / peak, 4)},
        "frac_of_peak": round(value / peak, 4),
        "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "step_ms": step_ms,
        "e2e": {"value": round(nbytes / (ms_e2e / 1e3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms_e2e, 4),
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 4},
        # route_pack, pack x, up/gate, pack h, down, combine
        "gpu_launches": 6 * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_config1_rate(args.cpu_seconds)
        except Exception as exc:
            line["cpu_baseline"] = {"value": None, "error": f"{type(exc).__name__}: {exc}"}
    if graph is not None:
        graph.reset()
    emit(line)


def cpu_config1_rate(seconds: float, sample_rows: int = 4):
    """The reference node's OpenMP FP8 CPU kernels at batch 1 on a sample of config-1 rows;
    the GB/s figure is config 1's algorithmic bytes over the extrapolated call time."""
    import numpy as np
    import torch

    from constellation_b200 import synthetic
    from oracle import refbuild

    threads = host_cores()
    kind = "reference" if refbuild.ref_available() else "port"
    n_e, row_slot, x, _ = config1_rows(torch)
    R = x.shape[0]
    xb = x.view(torch.int16).numpy().view(np.uint16)
    experts = {}
    starts = [0] + torch.cumsum(n_e, 0).tolist()[:-1]
    sample = [int(r) for r in starts[:sample_rows]]  # one row each of the first experts
    for r in sample:
        j = int(row_slot[r])
        if j not in experts:
            ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(j), device="cpu")
            experts[j] = refbuild.ExpertBytes(ex.w_up.numpy(), ex.s_up.numpy(), ex.w_gate.numpy(),
                                              ex.s_gate.numpy(), ex.w_down.numpy(), ex.s_down.numpy())

    def one(r):
        ex = experts[int(row_slot[r])]
        if kind == "reference":
            refbuild.ref_expert_cpu(ex, xb[r:r + 1], 2, 2, threads)
        else:
            xf = (xb[r].astype(np.uint32) << 16).view(np.float32)
            refbuild.oracle_expert_lut(ex, xf[None])

    one(sample[0])
    n = 0
    t0 = time.perf_counter()
    while True:
        for r in sample:
            one(r)
        n += len(sample)
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    ms_row = dt / n * 1e3
    ms_call = ms_row * R
    return {"value": round(config1_bytes(R) / (ms_call / 1e3) / 1e9, 4), "unit": "GB/s", "cores": threads,
            "threads": host_threads_note(threads), "kind": kind, "sample": f"{n} batch-1 expert calls over one row each of experts 0..{len(sample) - 1} ({dt:.1f} s); "
                                   f"one config-1 step = {R} such calls = {ms_call:.0f} ms (extrapolated)",
            "ms_per_row": round(ms_row, 2)}


# ---------------------------------------------------------------------------------------
W_EXPERTS = 32  # experts the node's requests cycle over: 1.41 GB of weights, more than L2


def worker_requests(torch, batch: int, seed: int = 0):
    """One seeded bf16 -> bf16 InferRequest body per resident expert (global ids 0..31),
    ``batch`` N(0, 1) rows each, and the rows themselves."""
    from constellation_b200 import protocol as P

    g = torch.Generator().manual_seed(seed)
    xs = torch.randn((W_EXPERTS, batch, H), generator=g).to(torch.bfloat16)
    bodies = [P.encode_infer_request(dict(expert_id=j, batch_size=batch, hidden_dim=H, input_dtype=2,
                                          output_dtype=2, activation=xs[j].view(torch.int16).numpy().tobytes()))
              for j in range(W_EXPERTS)]
    return xs, bodies


def worker_metric(batch: int) -> str:
    return f"expert requests/s (batch-{batch} bf16 InferRequest, one DeepSeek-V3 FP8 expert each)"


def run_worker(args):
    """The expert node's request path (``worker.cc`` HandleInferRequest + RunExpertRequest):
    a step is one request to each of 32 resident experts in turn.  ``value``: requests/s
    with the rows already on the device (``cst_expert_forward``); ``e2e``: the same
    requests as wire bodies through ``cst_serve_infer_request`` (decode, host-to-device
    copy, expert, device-to-host copy into the response body, encode, stream sync)."""
    import torch

    from constellation_b200 import protocol as P
    from constellation_b200 import synthetic
    from constellation_b200.context import ExpertContext, MoEConfig
    from constellation_b200.worker import handle_infer_request

    if int(os.environ.get("WORLD_SIZE", "1")) != 1 or args.gpus != 1:
        raise SystemExit("--workload worker is a single-GPU configuration")
    batch = int(args.tokens or 1)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = ExpertContext(dev, MoEConfig(), n_slots=W_EXPERTS, max_tokens=64, max_rows=max(batch, 64 * (K + 1)))
    for j in range(W_EXPERTS):
        ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(j), device=dev)
        ctx.upload_expert(j, j, ex.w_up, ex.s_up, ex.w_gate, ex.s_gate, ex.w_down, ex.s_down)
        del ex
    xs_h, bodies = worker_requests(torch, batch)
    xs = xs_h.to(dev)
    y = torch.empty((batch, H), dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize(dev)

    def step():
        for j in range(W_EXPERTS):
            ctx.expert_forward(j, xs[j], out=y)

    def timed(fn, k):
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b)

    for _ in range(max(3, args.warmup)):
        step()
    graph = None
    if not args.no_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(3):
            graph.replay()
    run = graph.replay if graph is not None else step
    with ClockSampler(smi_gpu_id(torch, dev)) as clk:
        ms_step = timed(run, args.steps) / args.steps
    clocks = clk.summary()
    ms_req = ms_step / W_EXPERTS

    # end to end: wire bodies in, wire bodies out, one synchronous request at a time
    def e2e_step():
        resp = None
        for body in bodies:
            resp = handle_infer_request([ctx], body)
        return resp

    for _ in range(3):
        last = e2e_step()
    r = P.decode_infer_response(last)
    if r["status_code"] != 0 or len(r["output"]) != batch * H * 2:
        raise RuntimeError(f"worker request failed: status {r['status_code']}")
    ms_e2e = timed(e2e_step, args.steps) / args.steps
    step_ms = step_distribution(torch, run, args.steps, dev)

    ctx.profile(True)
    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    stages = ctx.profile_read()
    ctx.profile(False)
    stage_ms = {k: statistics.mean(st[k] for st in stages) for k in stages[0]}
    req_bytes = EXPERT_BYTES + batch * H * (2 + 2)
    upg_ms, dn_ms = stage_ms["grouped_up_gate"], stage_ms["grouped_down"]
    peak, peak_kind = measured_peaks()
    ach = req_bytes / ((upg_ms + dn_ms) / 1e3) / 1e9
    line = {
        "metric": worker_metric(batch),
        "value": round(1e3 / ms_req, 1),
        "unit": "requests/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 weights x e4m3(3-term) activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, 128x128 block E4M3; N(0,1) bf16 rows)",
        "config": {"workload": f"worker_requests_batch{batch}", "experts": W_EXPERTS, "batch": batch,
                   "requests_per_step": W_EXPERTS, "hidden": H, "inter": I, "cuda_graph": graph is not None,
                   "l2": "no flush: the 32 experts' 1.41 GB of weights exceed the 126 MB L2"},
        "roofline": {"kernel": "grouped_ffn_tc up/gate + down of one request (tcgen05, TMA bulk ring)",
                     "bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach / peak, 4), "peak_source": peak_kind, "bytes_per_launch": req_bytes,
                     "ms_per_launch": round(upg_ms + dn_ms, 4), "traffic": None},
        "us_per_request": round(ms_req * 1e3, 2),
        "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "step_ms": step_ms,
        "e2e": {"value": round(W_EXPERTS * 1e3 / ms_e2e, 1), "unit": "requests/s",
                "us_per_request": round(ms_e2e * 1e3 / W_EXPERTS, 2),
                "h2d_bytes_per_step": W_EXPERTS * batch * H * 2, "d2h_bytes_per_step": W_EXPERTS * batch * H * 2,
                "path": "wire body -> cst_serve_infer_request -> wire body, synchronous per request"},
        # route_pack, pack x, up/gate, pack h, down, combine per request
        "gpu_launches": 6 * W_EXPERTS * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_worker_rate(args.cpu_seconds, batch)
        except Exception as exc:
            line["cpu_baseline"] = {"value": None, "error": f"{type(exc).__name__}: {exc}"}
    if graph is not None:
        graph.reset()
    emit(line)


def cpu_worker_rate(seconds: float, batch: int = 1, sample_experts: int = 4):
    """The reference node's OpenMP FP8 CPU kernels serving the same requests (one batch-1
    call per row, as RunExpertRequest takes batch 1) on a sample of the experts."""
    import numpy as np
    import torch

    from constellation_b200 import synthetic
    from oracle import refbuild

    threads = host_cores()
    kind = "reference" if refbuild.ref_available() else "port"
    xs, _ = worker_requests(torch, batch)
    experts = []
    for j in range(sample_experts):
        ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(j), device="cpu")
        experts.append(refbuild.ExpertBytes(ex.w_up.numpy(), ex.s_up.numpy(), ex.w_gate.numpy(), ex.s_gate.numpy(),
                                            ex.w_down.numpy(), ex.s_down.numpy()))
    xb = xs.view(torch.int16).numpy().view(np.uint16)

    def one(j):
        if kind == "reference":
            refbuild.ref_expert_cpu(experts[j], xb[j], 2, 2, threads)
        else:
            for row in xb[j]:
                xf = (row.astype(np.uint32) << 16).view(np.float32)
                refbuild.oracle_expert_lut(experts[j], xf[None])

    one(0)
    n = 0
    t0 = time.perf_counter()
    while True:
        for j in range(sample_experts):
            one(j)
        n += sample_experts
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": round(n / dt, 3), "unit": "requests/s", "cores": threads, "kind": kind,
            "threads": host_threads_note(threads),
            "sample": f"{n} batch-{batch} requests to experts 0..{sample_experts - 1} ({dt:.1f} s)",
            "ms_per_request": round(dt / n * 1e3, 2)}


# ---------------------------------------------------------------------------------------
class CpuReferenceLayer:
    """The reference CPU path for a sample of tokens: router (CPU restatement of
    route_token_real), one batch-1 call of the reference node's OpenMP FP8 expert kernels
    per (token, expert) and for the shared expert, fp32 combine (combine_outputs_torch)."""

    def __init__(self, sample_tokens: int, threads: int, zipf: bool = False):
        import numpy as np
        import torch

        from constellation_b200 import synthetic
        from oracle import refbuild

        self.np = np
        self.threads = threads
        self.kind = "reference" if refbuild.ref_available() else "port"
        self.refbuild = refbuild
        torch.manual_seed(0)
        gw, gb = synthetic.make_router(H, E, seed=synthetic.router_seed(), device="cpu")
        if zipf:
            gb = synthetic.zipf_bias(E, seed=synthetic.router_seed(), device="cpu")
        self.gw, self.gb = gw.numpy(), gb.numpy()
        x = synthetic.make_activations(sample_tokens, H, seed=synthetic.ACTIVATION_SEED, device="cpu")
        self.x_bits = x.view(torch.int16).numpy().view(np.uint16)
        self.x = x.float().numpy()
        from oracle import router as orouter

        self.orouter = orouter
        r = orouter.route_batched(self.x, self.gw, self.gb, n_group=G, topk_group=TG, top_k=K)
        need = sorted(set(int(e) for e in r.topk_idx.reshape(-1)))
        self.experts = {}
        for e in need + [-1]:
            ex = synthetic.make_expert(H, I, seed=synthetic.expert_seed(e), device="cpu")
            self.experts[e] = refbuild.ExpertBytes(ex.w_up.numpy(), ex.s_up.numpy(), ex.w_gate.numpy(),
                                                   ex.s_gate.numpy(), ex.w_down.numpy(), ex.s_down.numpy())
        self.sample_tokens = sample_tokens

    def run(self):
        np = self.np
        out = np.zeros((self.sample_tokens, H), np.float32)
        for t in range(self.sample_tokens):
            r = self.orouter.route_batched(self.x[t:t + 1], self.gw, self.gb, n_group=G, topk_group=TG, top_k=K)
            acc = np.zeros(H, np.float32)
            for e, w in zip(r.topk_idx[0], r.topk_weight[0]):
                y = self._expert(int(e), self.x_bits[t:t + 1])
                acc += np.float32(w) * y
            acc += self._expert(-1, self.x_bits[t:t + 1])
            out[t] = acc
        return out

    def _expert(self, e, xb):
        """One batch-1 expert call on bf16 bits ``xb [1, H]`` -> fp32 ``[H]``."""
        np = self.np
        ex = self.experts[e]
        if self.kind == "reference":
            yb = self.refbuild.ref_expert_cpu(ex, xb, 2, 2, self.threads)  # bf16 in, bf16 out
            return (yb[0].astype(np.uint32) << 16).view(np.float32)
        xf = (xb[0].astype(np.uint32) << 16).view(np.float32)
        _, y = self.refbuild.oracle_expert_lut(ex, xf[None])
        return y[0]


def cpu_reference_rate(sample_tokens: int, seconds: float, T: int = 64, zipf: bool = False):
    threads = host_cores()
    layer = CpuReferenceLayer(sample_tokens, threads, zipf=zipf)
    layer.run()  # warm-up (page in the weights)
    n = 0
    t0 = time.perf_counter()
    while True:
        layer.run()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    tok_s = n * sample_tokens / dt
    return {"value": round(tok_s, 3), "unit": "tokens/s", "cores": threads, "kind": layer.kind,
            "threads": host_threads_note(threads),
            "sample": f"{sample_tokens} tokens of the T={T} batch through router + 8 routed + shared experts at "
                      f"batch 1 per (token, expert), {n} repetitions, {dt:.1f} s",
            "ms_per_token": round(dt / (n * sample_tokens) * 1e3, 2)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "config1":
        base = cpu_config1_rate(args.cpu_seconds)
        emit({"impl": "reference", "metric": "expert-matvec HBM GB/s (grouped FP8 SwiGLU, 32 resident experts, "
              "n_e ~ U{1..16})", "value": base["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "dtype": "fp32 (FP8 LUT decode x block scale)", "data": "synthetic",
              "config": {"workload": "config1_grouped_matvec_32experts", "parallelism": "cpu"},
              "cpu_baseline": base,
              "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return
    if args.workload == "worker":
        batch = int(args.tokens or 1)
        base = cpu_worker_rate(args.cpu_seconds, batch)
        emit({"impl": "reference", "metric": worker_metric(batch), "value": base["value"], "unit": "requests/s",
              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
              "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (FP8 LUT decode x block scale)",
              "data": "synthetic", "config": {"workload": f"worker_requests_batch{batch}", "parallelism": "cpu"},
              "cpu_baseline": base,
              "e2e": {"value": base["value"], "unit": "requests/s", "h2d_bytes_per_step": 0,
                      "d2h_bytes_per_step": 0}})
        return
    if args.workload == "config3":
        # one token through one layer of the reference CPU path, times the layer count
        base = cpu_reference_rate(args.cpu_sample_tokens, args.cpu_seconds, T=args.tokens or 128)
        L, T3 = args.layers, args.tokens or 128
        v = base["value"] / L
        emit({"impl": "reference", "metric": f"MoE decode step tokens/s ({L} stacked DeepSeek-V3 MoE layers, "
              f"T={T3})", "value": round(v, 4), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
              "dtype": "fp32 (FP8 LUT decode x block scale)", "data": "synthetic",
              "config": {"workload": "config3_decode_stack" if L == 58 else f"config3_shape_{L}_layers",
                         "layers": L, "tokens": T3, "parallelism": "cpu"},
              "cpu_baseline": dict(base, value=round(v, 4),
                                   sample=base["sample"] + f"; per step x {L} layers (extrapolated)"),
              "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return
    threads = host_cores()
    prefill = args.workload == "config4"
    T = args.tokens or (4096 if prefill else 64)
    layer = CpuReferenceLayer(args.cpu_sample_tokens, threads, zipf=prefill)
    for _ in range(max(1, args.warmup)):
        layer.run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer.run()
    dt = time.perf_counter() - t0
    value = args.steps * args.cpu_sample_tokens / dt
    ms = dt / args.steps * 1e3
    line = {
        "impl": "reference",
        "metric": ("MoE-layer prefill tokens/s (1 DeepSeek-V3 MoE layer, T=4096, Zipf-skewed routing)" if prefill
                   else "MoE-layer decode tokens/s (1 DeepSeek-V3 MoE layer, T=64, 256 FP8 experts + shared)"),
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp32 (FP8 LUT decode x block scale)",
        "data": "synthetic (seeded N(0,0.02) weights, 128x128 block E4M3; RMS-normalised N(0,1) bf16 hidden)",
        "config": {"workload": "config4_prefill_T4096_one_layer" if prefill else "config2_decode_T64_one_layer",
                   "tokens": T, "routed_experts": E,
                   "shared_expert": True, "hidden": H, "inter": I, "top_k": K, "parallelism": "cpu",
                   "sample_tokens_per_step": args.cpu_sample_tokens},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": layer.kind,
                         "threads": host_threads_note(threads),
                         "sample": f"{args.cpu_sample_tokens} tokens of the T={T} batch per step, batch 1 "
                                   "per (token, expert) through the reference node's OpenMP FP8 CPU kernels"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


_RESULT_FD = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the original stdout."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _RESULT_FD
    args = parse()
    # Libraries (NCCL's banner, CUDA) may print to the C-level stdout; send all of that to
    # stderr so stdout carries only the result line.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config1":
        run_config1(args)
    elif args.workload == "config3":
        run_config3(args)
    elif args.workload == "worker":
        run_worker(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
