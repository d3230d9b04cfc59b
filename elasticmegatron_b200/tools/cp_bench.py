"""Context-parallel attention micro-benchmark: forward + backward of one attention layer, per CP exchange.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        -m elasticmegatron_b200.tools.cp_bench --seq 8192 --groups 32 --hpg 1 --iters 10

Each rank holds its two load-balanced chunks of the global sequence (chunks r and 2N-1-r); the time is the device
time of ``fn(qkv).backward(dout)`` (CUDA events, after warm-up), MAX over ranks, for ``all_gather``, ``p2p`` (ring)
and ``a2a`` (Ulysses), plus the same layer unsplit on one GPU for reference (rank 0 alone, whole sequence).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--groups", type=int, default=32)
    ap.add_argument("--hpg", type=int, default=1)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from elasticmegatron_b200.ops import functional as F_
    from elasticmegatron_b200.parallel.context_parallel import (cp_attention, cp_ring_attention,
                                                                cp_ulysses_attention)

    n, rank = dist.get_world_size(), dist.get_rank()
    S, b, G, hpg, d = a.seq, a.batch, a.groups, a.hpg, 128
    s = S // n
    qkv = torch.randn(s, b, G, hpg + 2, d, device="cuda").bfloat16()
    dout = torch.randn(s, b, G * hpg * d, device="cuda").bfloat16()
    fwd_flops = 4 * b * G * hpg * S * S * d / 2  # causal, whole sequence
    per_rank = 3.5 * fwd_flops / n  # forward + backward (2.5x the forward)
    rows = []
    for name, fn in (("all_gather", cp_attention), ("p2p", cp_ring_attention), ("a2a", cp_ulysses_attention)):
        if name == "a2a" and G % n:
            continue
        x = qkv.clone().requires_grad_()

        def step():
            x.grad = None
            fn(x, hpg, dist.group.WORLD, rank, n).backward(dout)

        ms = torch.tensor([_time(step, a.iters, a.warmup)], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        rows.append({"cp": n, "cp_comm_type": name, "seq": S, "heads": G * hpg, "kv_heads": G,
                     "ms_fwd_bwd": ms.item(), "tflops_per_gpu": per_rank / ms.item() / 1e9})
    if rank == 0:
        full = torch.randn(S, b, G, hpg + 2, d, device="cuda").bfloat16().requires_grad_()
        dfull = torch.randn(S, b, G * hpg * d, device="cuda").bfloat16()

        def step1():
            full.grad = None
            F_.attention(full, hpg).backward(dfull)

        ms1 = _time(step1, a.iters, a.warmup)
        rows.append({"cp": 1, "cp_comm_type": "none (one GPU, whole sequence)", "seq": S, "heads": G * hpg,
                     "kv_heads": G, "ms_fwd_bwd": ms1, "tflops_per_gpu": 3.5 * fwd_flops / ms1 / 1e9})
        for r in rows:
            print(json.dumps(r))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
