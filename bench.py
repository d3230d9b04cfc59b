"""Headline benchmark: Llama-2 7B bf16 training throughput (tokens/s per box) on N B200s, plus reshard latency.

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference ...                      # the reference's own build (unavailable offline)

N > 1 is launched by torchrun (one rank per GPU, NCCL).  Config (BASELINE config 2 shape): 32 layers, hidden
4096, 32 heads, ffn 11008, vocab 32000, seq 4096, micro-batch 1, global batch 16 per GPU (128 at 8 GPUs, weak
scaling), distributed Adam with fp32 master / moments, synthetic uniform token ids, N(0, 0.02) init.

Timing: W untimed steps, then exactly K steps bracketed by a barrier and ``cuda.synchronize`` on both sides and
timed with CUDA events on the compute stream; the value is the MAX over ranks.  Every step's inputs (~16 x 4 K
token ids per GPU, 1 MiB) come from pinned host memory, and the activations / weights (>100 GB) dwarf the
126 MB L2, so no L2 flush is needed.  A second loop of K steps through the same public call with the loss read
back to the host every step gives the end-to-end figure.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "reshard latency ms (p50) + tokens/s/box per strategy at 1/2/4/8 B200, max over ranks"


def _clock_sampler(dev_index: int, stop: threading.Event, out: list):
    try:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        out.append(("max", mx))
        while not stop.is_set():
            sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
            try:
                rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                rs = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
            util = pynvml.nvmlDeviceGetUtilizationRates(h).gpu
            out.append((sm, rs, util))
            stop.wait(0.2)
    except Exception as e:  # pragma: no cover
        out.append(("error", repr(e)))


_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost"}


def _summarize_clocks(samples: list) -> dict:
    mx = next((v for k, v in samples if k == "max"), None) if samples and isinstance(samples[0], tuple) else None
    rows = [s for s in samples if len(s) == 3]
    loaded = [s for s in rows if s[2] >= 50] or rows
    reasons = set()
    for _, rs, _ in loaded:
        for bit, name in _REASONS.items():
            if rs & bit:
                reasons.add(name)
    sm = statistics.median([s[0] for s in loaded]) if loaded else None
    return {"sm_mhz": sm, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(rows)}


def reference_arm(args):
    print(json.dumps({"impl": "reference", "unavailable": (
        "the reference (infinigence/ElasticMegatron) is a plug-in for Megatron-LM core_r0.11 + TransformerEngine, "
        "neither of which is installed or installable offline; the reference source tree has no setup.py / pyproject.toml, so "
        "pip cannot install it either")}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="own", choices=["own", "reference"])
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--layers", type=int, default=None, help="(debug only) override the layer count")
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--per-gpu-batch", type=int, default=16)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--reshard-iters", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    from elasticmegatron_b200.config import Args, TrainConfig, preset, set_args
    from elasticmegatron_b200.ops.native import ext, launch_count
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    ext()
    over = {}
    if args.layers:
        over["num_layers"] = args.layers
    if args.seq:
        over["seq_length"] = args.seq
    cfg = preset(args.model, max_tensor_parallel_size=8, **over)
    gbs = args.per_gpu_batch * world
    tc = TrainConfig(micro_batch_size=1, global_batch_size=gbs, lr=3e-4, min_lr=3e-5, lr_warmup_iters=2,
                     train_iters=1000, overlap_grad_reduce=world > 1, seed=0)
    set_args(Args(model=cfg, train=tc))
    tp, pp = args.tp, args.pp
    strat = dict(world_size=world, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp)
    S = ParallelStrategy(**strat)
    par = f"tp{tp}" * (tp > 1) + f"pp{pp}" * (pp > 1) + f"dp{S.data_parallel_size}"
    alt = None
    strategies = [strat]
    if world > 1 and tp == 1 and pp == 1:
        alt = dict(world_size=world, tensor_model_parallel_size=2, pipeline_model_parallel_size=1)
        strategies.append(alt)
    if world > 1:
        create_all_groups([ParallelStrategy(**s) for s in strategies])
    ts = TrainingState(S)
    ts.init_weights(0, method="local")
    it = DataloaderState.build_iterators(ts, 0)[0]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        train_step(ts, it, return_loss=False)
    barrier()
    samples, stop = [], threading.Event()
    th = threading.Thread(target=_clock_sampler, args=(local, stop, samples), daemon=True)
    th.start()
    time.sleep(0.3)
    n0 = launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(args.steps):
        train_step(ts, it, return_loss=False)
    e1.record()
    barrier()
    launches = launch_count() - n0
    ms = e0.elapsed_time(e1)
    # end-to-end through the public call: pinned-host inputs copied every step, loss read back every step
    e2e_ms = None
    loss = None
    if not args.no_e2e:
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            loss = train_step(ts, it, return_loss=True)["loss"]
        barrier()
        e2e_ms = (time.perf_counter() - t0) * 1e3
    stop.set()
    th.join(timeout=2)
    vals = torch.tensor([ms, e2e_ms or 0.0, float(launches)], device="cuda")
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms_max, launches = vals.tolist()
    tokens_per_step = gbs * cfg.seq_length
    value = tokens_per_step * args.steps / (ms / 1e3)

    # reshard latency (multi-GPU): alternate between the benchmark layout and TP2
    reshard = None
    if alt is not None and args.reshard_iters > 0:
        try:
            from elasticmegatron_b200.runtime.manager import ElasticMegatronManager

            mgr = ElasticMegatronManager(strategies, training_state=ts, engine="native")
            lat = []
            for i in range(args.reshard_iters * 2):
                ts2 = mgr.reshard(strategies[(i + 1) % 2])
                lat.append(mgr.last_switch["transfer_ms"])
            reshard = {"p50_ms": statistics.median(lat), "all_ms": lat, "gbytes": mgr.last_switch["gbytes"],
                       "nvlink_roofline_ms": mgr.last_switch["nvlink_roofline_ms"],
                       "pair": [str(ParallelStrategy(**s)) for s in strategies]}
        except Exception as e:  # report, never crash the throughput line
            reshard = {"error": repr(e)[:300]}
    if rank == 0:
        h2d = args.per_gpu_batch * cfg.seq_length * 8 * 2 * world  # ids + labels, int64
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids, random N(0,0.02) init)",
            "config": {"model": args.model + (f"-{cfg.num_layers}L" if args.layers else ""), "global_batch": gbs,
                       "seq_len": cfg.seq_length, "parallelism": par, "micro_batch": 1,
                       "l2": "inputs+weights far larger than L2 (no flush needed)"},
            "clocks": _summarize_clocks(samples),
            "e2e": {"value": tokens_per_step * args.steps / (e2e_ms_max / 1e3) if e2e_ms else None,
                    "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * world,
                    "loss": loss},
            "gpu_launches": int(launches),
            "reshard": reshard,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
