"""All-reduce micro-benchmark: NCCL against the symmetric-memory reducers (NVSwitch multicast and peer memory).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        -m elasticmegatron_b200.tools.comm_bench --sizes-mb 16,64,256 --iters 20

Device time per call (CUDA events on the launching stream, after warm-up), MAX over ranks.  Bus bandwidth uses
the ring convention 2 (n - 1) / n * bytes / time, so the figures compare with nccl-tests' busbw.  Each result is
checked against NCCL's.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def run(group, sizes_mb, iters: int = 20, warmup: int = 5):
    """Time NCCL, the multicast and the peer-memory all-reduce over ``group`` (every rank calls it); returns one
    row per (implementation, size) with device ms (MAX over ranks), bandwidths and a check against NCCL."""
    from elasticmegatron_b200.parallel import nvls

    n, rank = dist.get_world_size(group), dist.get_rank(group)
    dev = torch.device("cuda", torch.cuda.current_device())
    chunk = max(sizes_mb) << 20
    reducers = {"nvls": nvls.SymmetricAllReduce(group, dev, chunk_bytes=chunk),
                "p2p": nvls.SymmetricAllReduce(group, dev, chunk_bytes=chunk, force_p2p=True)}
    rows = []
    for mb in sizes_mb:
        numel = (mb << 20) // 4
        x0 = torch.randn(numel, device=dev, generator=torch.Generator(device=dev).manual_seed(rank))
        ref = x0.clone()
        dist.all_reduce(ref, group=group)
        impls = {"nccl": lambda t: dist.all_reduce(t, group=group)}
        for k, r in reducers.items():
            if k == "nvls" and r.kind != "nvls":
                continue
            impls[k] = r.all_reduce_
        for name, fn in impls.items():
            x = x0.clone()
            fn(x)
            torch.cuda.synchronize()
            ok = bool(torch.allclose(x, ref, rtol=1e-5, atol=1e-5))
            for _ in range(warmup):
                fn(x)
            dist.barrier(group=group)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn(x)
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / iters], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=group)
            t = ms.item()
            nbytes = numel * 4
            rows.append({"impl": name, "n_gpus": n, "mbytes": mb, "ms": t, "algbw_gbs": nbytes / t / 1e6,
                         "busbw_gbs": 2 * (n - 1) / n * nbytes / t / 1e6, "matches_nccl": ok})
        del x0, ref, x
    # nobody frees its staging buffer while a peer may still touch it
    torch.cuda.synchronize()
    dist.barrier(group=group)
    reducers.clear()
    torch.cuda.synchronize()
    dist.barrier(group=group)
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="16,64,256")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    g = dist.new_group(list(range(dist.get_world_size())))
    rows = run(g, [int(x) for x in a.sizes_mb.split(",")], a.iters, a.warmup)
    if dist.get_rank() == 0:
        for r in rows:
            print(json.dumps(r))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
