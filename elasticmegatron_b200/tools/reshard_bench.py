"""Reshard microbenchmark: switch latency, bytes moved and NVLink-roofline fraction.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m elasticmegatron_b200.tools.reshard_bench \
        --model llama2-13b --engines native,torch --pairs all --alternate 20

State per rank: the bf16 parameter arena and the fp32 ``[3, n]`` optimizer arena (master / exp_avg /
exp_avg_sq) of the source and destination layouts - exactly what a switch moves; no model or gradient
buffers are built.  Values are N(0, 0.02) parameters (master = param) and moments uniform in [0, 1e-3).

For every ordered pair of strategies the engine runs ``--iters`` timed switches after one warm-up switch
(which maps peer memory and builds the task table); each switch is timed with CUDA events on the compute
stream (the engine's own stream-ordered barriers included) and the MAX over ranks is reported.  The roofline
is max over GPUs of max(egress, ingress) non-local bytes / ``--link-gbs`` (measured peer-copy bandwidth per
direction).  ``reference`` runs the reference's three-phase per-(param, tensor, peer) blocking schedule
followed by bf16 regeneration from the master and a DP all-gather, as the reference does.
"""
from __future__ import annotations

import argparse
import itertools
import json
import os
import statistics

import numpy as np
import torch
import torch.distributed as dist


def _strategies(world):
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy

    out = []
    for tp in (1, 2, 4, 8):
        for pp in (1, 2, 4, 8):
            if world % (tp * pp) == 0:
                out.append(ParallelStrategy(world_size=world, tensor_model_parallel_size=tp,
                                            pipeline_model_parallel_size=pp))
    return out


def _fill(param, opt, rl, seed, rank):
    """Params N(0, 0.02); master = the own shard of the params; moments uniform in [0, 1e-3)."""
    g = torch.Generator(device=param.device)
    g.manual_seed(seed * 131 + rank)
    param.normal_(0.0, 0.02, generator=g)
    for a, e, o in rl.owned():
        opt[0, o:o + (e - a)].copy_(param[a:e].float())
    opt[1:].uniform_(0.0, 1e-3, generator=g)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama2-13b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--engines", default="native")
    ap.add_argument("--pairs", default="all", help="'all' or a comma list like tp1pp1-tp4pp1")
    ap.add_argument("--alternate", type=int, default=20, help="TP1*DP8 <-> TP4*DP2 switches (0 = skip)")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--link-gbs", type=float, default=900.0, help="link rate per direction (nominal NVLink 5: 900 GB/s; pass a measured rate to compare)")
    ap.add_argument("--out", default=None)
    ap.add_argument("--mode", default="push", choices=["pull", "push"], help="native engine: who runs each copy")
    args = ap.parse_args()

    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)
    from elasticmegatron_b200.config import Args, TrainConfig, preset, set_args
    from elasticmegatron_b200.parallel.process_groups import ParallelState, ProcessGroupPool, create_all_groups
    from elasticmegatron_b200.planner.layout import rank_layout
    from elasticmegatron_b200.planner.plan import build_plan
    from elasticmegatron_b200.runtime.memory import get_pool
    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine
    from elasticmegatron_b200.transfer.reference_engine import ReferenceAlgorithmEngine
    from elasticmegatron_b200.transfer.torch_engine import TorchP2PEngine

    over = {"num_layers": args.layers} if args.layers else {}
    cfg = preset(args.model, max_tensor_parallel_size=8, **over)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True)))
    S = _strategies(world)
    create_all_groups(S)
    pool = get_pool(dev)

    def arenas(s):
        rl = rank_layout(cfg, s, rank, True, None)
        pa = pool.alloc(rl.param_numel * 2)
        oa = pool.alloc(rl.opt_numel * 12)
        return pa, oa, pa.view(torch.bfloat16, (rl.param_numel,)), oa.view(torch.float32, (3, rl.opt_numel)), rl

    def regen_allgather(s, P, O, rl):
        """The reference's bf16 regeneration from the master + DP all-gather (training_state.py:176-197)."""
        for a, e, o in rl.owned():
            P[a:e].copy_(O[0, o:o + (e - a)].to(P.dtype))
        ps = ParallelState(s)
        for kind, bl, base, gname in (("d", rl.dense, 0, "zero"), ("e", rl.expert, rl.dense.numel, "expert_zero")):
            if bl is None:
                continue
            n = len(ps.group_ranks[gname])
            z = rl.dense_shard_index if kind == "d" else rl.expert_shard_index
            for bs, be in bl.buckets:
                buf = P[base + bs:base + be]
                c = buf.numel() // n
                if n > 1:
                    dist.all_gather_into_tensor(buf, buf[z * c:(z + 1) * c].clone(), group=ps.groups[gname])

    if args.pairs == "all":
        pairs = list(itertools.permutations(S, 2))
    else:
        names = {f"tp{s.tensor_model_parallel_size}pp{s.pipeline_model_parallel_size}": s for s in S}
        pairs = [(names[a], names[b]) for a, b in (p.split("-") for p in args.pairs.split(","))]
    engines = {"native": NativeP2PEngine, "torch": TorchP2PEngine, "reference": ReferenceAlgorithmEngine}
    results = []

    def fits(a, b) -> bool:
        """Source and destination arenas (params + optimizer) of the largest rank must fit together."""
        need = 0
        for r in range(max(a.world_size, b.world_size)):
            n = 0
            for s in (a, b):
                if r < s.world_size:
                    rl = rank_layout(cfg, s, r, True, None)
                    n += rl.param_numel * 2 + rl.opt_numel * 12
            need = max(need, n)
        return need * 1.05 < torch.cuda.get_device_properties(dev).total_memory

    def run_pair(eng_name, eng, a, b, iters):
        plan = build_plan(a, b, cfg, overlap_grad_reduce=True, ddp_bucket_size=None)
        sa = arenas(a) if rank < a.world_size else None
        sb = arenas(b) if rank < b.world_size else None
        if sa:
            _fill(sa[2], sa[3], sa[4], 1, rank)
        union = sorted(set(range(a.world_size)) | set(range(b.world_size)))
        group = ProcessGroupPool.get(union)
        times = []
        for i in range(iters + 1):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            eng.execute(plan, rank, sa[2] if sa else None, sa[3] if sa else None, sb[2] if sb else None,
                        sb[3] if sb else None, group)
            if eng_name == "reference" and sb:
                regen_allgather(b, sb[2], sb[3], sb[4])
            e1.record()
            torch.cuda.synchronize()
            if i > 0:
                times.append(e0.elapsed_time(e1))
        t = torch.tensor(times, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        m = plan.bytes_matrix(4, 2)
        np.fill_diagonal(m, 0)
        roof = plan.nvlink_roofline_ms(args.link_gbs, 4, 2)
        for x in (sa, sb):
            if x:
                pool.free(x[0])
                pool.free(x[1])
        return t.tolist(), int(m.sum()), roof

    for eng_name in args.engines.split(","):
        eng = engines[eng_name](mode=args.mode) if eng_name == "native" else engines[eng_name]()
        for a, b in pairs:
            if not fits(a, b):
                if rank == 0:
                    print(json.dumps({"engine": eng_name, "src": str(a), "dst": str(b), "skipped":
                                      "source and destination state do not fit in one GPU's memory together "
                                      "(use --layers to shrink the model)"}), flush=True)
                continue
            ts, nbytes, roof = run_pair(eng_name, eng, a, b, args.iters)
            p50 = statistics.median(ts)
            rec = {"engine": eng_name + (f"-{args.mode}" if eng_name == "native" else ""), "src": str(a), "dst": str(b), "p50_ms": p50, "all_ms": ts,
                   "bytes_moved": nbytes, "roofline_ms": roof, "roofline_frac": (roof / p50) if p50 else None}
            results.append(rec)
            if rank == 0:
                print(json.dumps(rec), flush=True)
        if args.alternate:
            x = next(s for s in S if s.tensor_model_parallel_size == 1 and s.pipeline_model_parallel_size == 1)
            y = next((s for s in S if s.tensor_model_parallel_size == 4 and s.pipeline_model_parallel_size == 1), None)
            if y is not None:
                lat, roofs = [], []
                for i in range(args.alternate):
                    a, b = (x, y) if i % 2 == 0 else (y, x)
                    ts, nbytes, roof = run_pair(eng_name, eng, a, b, 1)
                    lat.append(ts[0])
                    roofs.append(roof)
                p50 = statistics.median(lat)
                rec = {"engine": eng_name, "alternation": f"{x} <-> {y}", "p50_ms": p50, "all_ms": lat,
                       "roofline_ms": statistics.median(roofs), "roofline_frac": statistics.median(roofs) / p50}
                results.append(rec)
                if rank == 0:
                    print(json.dumps(rec), flush=True)
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
