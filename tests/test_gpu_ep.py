"""Expert parallelism over NCCL on 2 GPUs (skipped with fewer than 2 visible GPUs).

Each rank holds E/2 experts and the shared expert; tokens are split in half.  Both
exchange strategies must reproduce the single-process CPU oracle of the whole layer
within the layer tolerance (row-wise relative 2e-3 on fp32 outputs).  Ranks run as
spawned child processes with a 60 s process-group timeout; NVLS is off.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, H, I, G, TG, K = 16, 256, 128, 4, 2, 4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from constellation_b200.context import ExpertContext, MoEConfig
        from constellation_b200.ep import ExpertParallelMoE
        from oracle import cases

        T = 5 * world
        cfg = MoEConfig(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, n_group=G, topk_group=TG,
                        num_experts_per_tok=K)
        epr = E // world
        ctx = ExpertContext(dev, cfg, n_slots=epr + 3, max_tokens=T)
        for j in range(epr):
            e = rank * epr + j
            ctx.upload_bundle(j, e, cases.expert(3000 + e, H, I))
        ctx.upload_bundle(epr, -1, cases.expert(3999, H, I))
        w, b = cases.router(81, E, H, bias_std=0.05)
        gw, gb = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
        x = torch.from_numpy(cases.activations(82, T, H)).to(dev, torch.bfloat16)
        Tl = T // world
        xl = x[rank * Tl:(rank + 1) * Tl].contiguous()
        res = {}
        for mode in ("allgather", "allgather_local", "alltoall", "p2p", "p2p_replicated", "allgather_replicated"):
            if mode == "p2p_replicated":
                # experts 1 and E-2 replicated on every rank (the copies go to spare slots) and
                # served by each rank for its own tokens only: the same rows, spread differently
                reps = [e for e in (1, E - 2) if not (rank * epr <= e < (rank + 1) * epr)]
                for j, e in enumerate(reps):
                    ctx.upload_bundle(epr + 1 + j, e, cases.expert(3000 + e, H, I))
                for e in (1, E - 2):
                    ctx.set_own_tokens_only(e, True)
            base_mode = mode.split("_")[0]
            # allgather_local: own-token routing + gathered routes (the prefill-sized path)
            local = mode == "allgather_local"
            moe = ExpertParallelMoE(ctx, rank=rank, world=world, n_routed_experts=E,
                                    mode=base_mode, local_route_min=1 if local else 128)
            res[mode] = moe.forward(xl, gw, gb, out_dtype=torch.float32).cpu().numpy()
            if base_mode == "p2p":
                # a second exchange through the same buffers (epoch 2), then release them
                res[mode + "_again"] = moe.forward(xl, gw, gb, out_dtype=torch.float32).cpu().numpy()
                torch.cuda.synchronize()
                dist.barrier()
                moe.close()
        torch.cuda.synchronize()
        ctx.device_error()
        q.put((rank, res))
    except Exception as exc:  # report, then leave the group cleanly
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_both_modes():
    """Every exchange mode over 2 ranks (or 4 / 8 when the box has them) against the oracle."""
    n_dev = torch.cuda.device_count()
    if n_dev < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from oracle import cases
    from oracle.expert import DequantExpert
    from oracle.layer import moe_layer

    world = 8 if n_dev >= 8 else (4 if n_dev >= 4 else 2)
    T = 5 * world
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert isinstance(got[r], dict), got[r]
    w, b = cases.router(81, E, H, bias_std=0.05)
    x = cases.activations(82, T, H)
    ref = moe_layer(x, w, b, {e: DequantExpert(cases.expert(3000 + e, H, I)) for e in range(E)},
                    DequantExpert(cases.expert(3999, H, I)), n_group=G, topk_group=TG, top_k=K)
    for mode in ("allgather", "allgather_local", "alltoall", "p2p", "p2p_again", "p2p_replicated",
                 "p2p_replicated_again", "allgather_replicated"):
        out = np.concatenate([got[r][mode] for r in range(world)])
        num = np.abs(out - ref.out_f32).max(axis=1)
        den = np.abs(ref.out_f32).max(axis=1)
        assert float((num / den).max()) < 2e-3, mode
    # routing locally and gathering the routes gives the same routes, hence the same bits;
    # with two ranks the pushed partials add like the reduce-scatter's (one fp32 addition)
    for r in range(world):
        assert np.array_equal(got[r]["allgather"], got[r]["allgather_local"])
        assert np.array_equal(got[r]["p2p"], got[r]["p2p_again"])
        if world == 2:
            assert np.array_equal(got[r]["allgather"], got[r]["p2p"])
