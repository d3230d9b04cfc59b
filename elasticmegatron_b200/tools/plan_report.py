"""What a switch will move, before running it: bytes per GPU pair, the NVLink roofline, the per-parameter plan.

    python -m elasticmegatron_b200.tools.plan_report --model llama2-13b ws8 ws8-tp4
    python -m elasticmegatron_b200.tools.plan_report --model mixtral-8x7b --layers 2 ws8-ep8 ws8-tp2-ep4-etp1 --params

Runs the planner on the host only (no GPU, no processes).  The roofline is max over GPUs of max(egress, ingress)
bytes that cross NVLink divided by ``--link-gbs`` (default: the nominal 900 GB/s per direction of B200 peer
copies); the JSON line at the end holds the same figures, plus the host cost of a first switch between the
pair: building the plan (``plan_ms``, layouts not cached) and the slowest rank's transfer task table
(``tasks_ms_max``, with stand-in addresses).  Later switches between the same pair reuse both.
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def report(model: str, src: str, dst: str, layers=None, link_gbs: float = 900.0, params: bool = False,
           max_params=None) -> dict:
    from ..config import Args, TrainConfig, preset, set_args
    from ..parallel.strategy import ParallelStrategy
    from ..planner.plan import build_plan

    over = {"max_tensor_parallel_size": 8}
    if layers:
        over["num_layers"] = layers
    cfg = preset(model, **over)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True)))
    import time

    from ..planner import layout as _layout
    from ..transfer.native_engine import NativeP2PEngine

    a, b = ParallelStrategy.parse(src), ParallelStrategy.parse(dst)
    _layout._RL_CACHE.clear()
    t0 = time.perf_counter()
    plan = build_plan(a, b, cfg, overlap_grad_reduce=True, ddp_bucket_size=None)
    plan_ms = (time.perf_counter() - t0) * 1e3
    n = max(a.world_size, b.world_size)
    addrs = {r: tuple((1 << 40) * (4 * r + j + 1) for j in range(4)) for r in range(n)}  # stand-ins, never used
    eng, tasks_ms = NativeP2PEngine(), 0.0
    for r in range(n):
        t0 = time.perf_counter()
        eng._tasks(plan, r, addrs, 2)
        tasks_ms = max(tasks_ms, (time.perf_counter() - t0) * 1e3)
    dt = 4
    m = plan.bytes_matrix(dt, 2)
    local = int(np.trace(m))
    np.fill_diagonal(m, 0)
    out = {"model": model, "src": str(a), "dst": str(b), "copies": int(len(plan.desc)),
           "nvlink_bytes": int(m.sum()), "local_bytes": local,
           "max_egress_bytes": int(m.sum(1).max(initial=0)), "max_ingress_bytes": int(m.sum(0).max(initial=0)),
           "roofline_ms": plan.nvlink_roofline_ms(link_gbs, dt, 2), "link_gbs": link_gbs,
           "bytes_matrix_gb": (m / 1e9).round(3).tolist(), "plan_ms": plan_ms, "tasks_ms_max": tasks_ms,
           # same layout (only SP differs): the manager hands the arenas over instead of running the plan
           "handover": a.layout_key() == b.layout_key()}
    from ..planner.memory import layout_report, switch_peak_bytes

    out["memory_gb"] = {"src": {k: v / 1e9 for k, v in layout_report(cfg, a).items()},
                        "dst": {k: v / 1e9 for k, v in layout_report(cfg, b).items()},
                        "switch_peak_state": switch_peak_bytes(cfg, a, b) / 1e9}
    if params:
        out["plan"] = plan.describe(cfg, max_params=max_params)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--link-gbs", type=float, default=900.0, help="link rate per direction (nominal NVLink 5: 900 GB/s; pass a measured rate to compare)")
    ap.add_argument("--params", action="store_true", help="also print the per-parameter plan")
    ap.add_argument("--max-params", type=int, default=None)
    a = ap.parse_args(argv)
    r = report(a.model, a.src, a.dst, a.layers, a.link_gbs, a.params, a.max_params)
    print(f"{r['src']} -> {r['dst']} ({r['model']}): {r['copies']} copies, "
          f"{r['nvlink_bytes'] / 1e9:.2f} GB over NVLink, {r['local_bytes'] / 1e9:.2f} GB local; "
          f"busiest GPU sends {r['max_egress_bytes'] / 1e9:.2f} GB / receives {r['max_ingress_bytes'] / 1e9:.2f} GB; "
          f"NVLink roofline {r['roofline_ms']:.2f} ms at {r['link_gbs']:.0f} GB/s; host: plan {r['plan_ms']:.0f} ms, "
          f"task table {r['tasks_ms_max']:.0f} ms (slowest rank)")
    if r["handover"]:
        print("same layout (the strategies differ only in sequence parallelism): a switch hands the arenas over; "
              "nothing is copied")
    mem = r["memory_gb"]
    print(f"per-GPU memory (largest rank): source {mem['src']['peak']:.1f} GB (state {mem['src']['total']:.1f} + "
          f"activations ~{mem['src']['activations']:.1f}), destination {mem['dst']['peak']:.1f} GB; during the "
          f"switch both states: {mem['switch_peak_state']:.1f} GB")
    print("GB sent (row) -> received (column):")
    for i, row in enumerate(r["bytes_matrix_gb"]):
        print(f"  {i}: " + " ".join(f"{x:7.2f}" for x in row))
    if "plan" in r:
        print(r.pop("plan"))
    print(json.dumps({k: v for k, v in r.items() if k != "bytes_matrix_gb"}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
