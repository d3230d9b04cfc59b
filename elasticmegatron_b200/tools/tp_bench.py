"""Per-op benchmark of the fused tensor-parallel kernels against "GEMM + NCCL collective".

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m elasticmegatron_b200.tools.tp_bench --model llama2-7b

For every sequence-parallel linear of one transformer layer (QKV and fc1: all-gather -> GEMM; proj and fc2:
GEMM -> reduce-scatter; forward and the matching dgrad of the backward) it times, with CUDA events on the
compute stream after warm-up, the MAX over ranks of

* ``fused``: ``tp_fused.all_gather_gemm`` / ``tp_fused.gemm_reduce_scatter`` (one tcgen05 GEMM launch that
  moves the data over NVLink peer memory, plus its barrier / local reduction);
* ``nccl``: NCCL ``all_gather_into_tensor`` / ``reduce_scatter_tensor`` around the same tcgen05 GEMM;
* ``gemm``: the GEMM alone (the compute floor).

The roofline of a fused op is max(FLOPs / measured bf16 GEMM peak, bytes crossing NVLink per GPU / the link rate (nominal 900 GB/s per direction)).
Activations are larger than L2 for the default shapes (tokens = 4096).
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
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--tokens", type=int, default=4096, help="sequence length x micro-batch")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--peak-tflops", type=float, default=None)
    ap.add_argument("--link-gbs", type=float, default=900.0, help="link rate per direction (nominal NVLink 5: 900 GB/s; pass a measured rate to compare)")
    a = ap.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from ..config import preset
    from ..ops import tp_fused
    from ..ops.native import ext

    peak = a.peak_tflops
    if peak is None:
        try:
            with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
                peak = float(json.load(f)["bf16_tflops"])
        except Exception:
            peak = 1590.0
    cfg = preset(a.model)
    tp = dist.get_world_size()
    g = dist.group.WORLD
    rank = dist.get_rank()
    h, f = cfg.hidden_size, cfg.ffn_hidden_size
    kv = cfg.num_query_groups * (h // cfg.num_attention_heads)
    T = a.tokens
    torch.manual_seed(rank)
    dev = "cuda"
    qkv_out = (h + 2 * kv) // tp
    cases = [  # name, kind, rows of the full GEMM, K, N (per-rank weight [N, K] or [K, N])
        ("qkv.fwd", "ag", h, qkv_out), ("fc1.fwd", "ag", h, 2 * f // tp),
        ("proj.fwd", "rs", h // tp, h), ("fc2.fwd", "rs", f // tp, h),
        ("proj.dgrad", "ag_dgrad", h, h // tp), ("fc2.dgrad", "ag_dgrad", h, f // tp),
        ("qkv.dgrad", "rs_dgrad", qkv_out, h), ("fc1.dgrad", "rs_dgrad", 2 * f // tp, h),
    ]
    out = []
    for name, kind, K, N in cases:
        if kind in ("ag", "ag_dgrad"):
            shard = torch.randn(T // tp, K, device=dev).bfloat16()
            # fwd: x @ W^T with W [N, K]; dgrad of a row-parallel layer: dy @ W with W [K_out=K, N]
            w = (torch.randn(N, K, device=dev) if kind == "ag" else torch.randn(K, N, device=dev)).bfloat16()
            trans_b = kind == "ag"
            full = torch.empty(T, K, device=dev, dtype=torch.bfloat16)

            def fused():
                tp_fused.all_gather_gemm(shard, w, trans_b, g)

            def nccl():
                dist.all_gather_into_tensor(full, shard, group=g)
                ext().gemm_tc(full, w, False, trans_b)

            def gemm_only():
                ext().gemm_tc(full, w, False, trans_b)

            link_bytes = (tp - 1) * shard.numel() * 2
        else:
            x = torch.randn(T, K, device=dev).bfloat16()
            w = (torch.randn(N, K, device=dev) if kind == "rs" else torch.randn(K, N, device=dev)).bfloat16()
            trans_b = kind == "rs"
            red = torch.empty(T // tp, N, device=dev, dtype=torch.bfloat16)

            def fused():
                tp_fused.gemm_reduce_scatter(x, w, False, trans_b, g)

            def nccl():
                y = ext().gemm_tc(x, w, False, trans_b)
                dist.reduce_scatter_tensor(red, y, group=g)

            def gemm_only():
                ext().gemm_tc(x, w, False, trans_b)

            link_bytes = (tp - 1) * (T // tp) * N * 2
        flops = 2.0 * T * K * N
        t_f = _time(fused, a.iters, a.warmup)
        t_n = _time(nccl, a.iters, a.warmup)
        t_g = _time(gemm_only, a.iters, a.warmup)
        roof = max(flops / (peak * 1e12), link_bytes / (a.link_gbs * 1e9)) * 1e3
        rec = {"op": name, "tp": tp, "M": T, "K": K, "N": N, "fused_ms": t_f, "nccl_ms": t_n, "gemm_ms": t_g,
               "fused_speedup": t_n / t_f, "roofline_ms": roof, "fused_roofline_frac": roof / t_f,
               "fused_tflops": flops / t_f / 1e9}
        out.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)
    assert ext().comm_error_flag() == 0 and ext().gemm_error_flag() == 0
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
