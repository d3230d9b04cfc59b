"""Headline benchmark: Llama-2 7B bf16 training throughput (tokens/s per box) on N B200s, per strategy, plus the
latency of switching between those strategies.

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference ...                      # the reference's own build (unavailable offline)

N > 1 is launched by torchrun (one rank per GPU, NCCL).  Config: 32 layers, hidden 4096, 32
heads, ffn 11008, vocab 32000, seq 4096, micro-batch 1, global batch 16 per GPU (128 at 8 GPUs, weak scaling),
distributed Adam with fp32 master / moments, synthetic uniform token ids, N(0, 0.02) init.

Phases (all device times are CUDA events on the compute stream, MAX over ranks):

1. ``value``: W untimed steps, then exactly K steps under TP1 * DP N (``--tp/--pp`` pick another layout),
   bracketed by a barrier and ``cuda.synchronize`` on both sides.  The activations / weights (>100 GB) dwarf the
   126 MB L2, so no L2 flush is needed.
2. ``e2e``: K more steps through the same public call (``train_step``) with every step's token ids copied from
   pinned host memory and the loss read back to the host, timed by the host clock.
3. (N > 1) ``strategies``: the switching schedule of BASELINE config 2 scaled to N GPUs (at 8: TP8 -> TP4*DP2 ->
   TP2*PP2*DP2 -> TP1*DP8, sequence parallelism on whenever TP > 1): switch with the native engine, run one
   untimed step, then time ``--strategy-steps`` steps -> tokens/s per strategy (released state arenas are handed
   back to the driver first when less than a quarter of the GPU is free, so the step's activations fit).
4. (N > 1) ``switches``: for every consecutive pair of the schedule, ``--reshard-iters`` round trips without
   training in between; p50 device latency per direction, GB moved, and the roofline fraction at the nominal
   900 GB/s per direction and at the peer-copy rate measured at the start of this phase (``link_gbs_measured``,
   the K1 kernel pushing 1 GiB to the next rank, all ranks at once).  Before the first and after every switch a
   layout-independent, position-sensitive checksum of the whole model state (``transfer/validate.py``) must
   equal the one taken before the pair's switches: ``checksum_ok``.
5. (N > 1) ``context_engines``: the first pair once more with this repository's batched-NCCL engine and with
   its re-implementation of the reference's transfer schedule (both repo code, labelled as such; they are not
   the reference's own build).
6. (N > 1) ``allreduce_256mb``: a 256 MB fp32 all-reduce over all N GPUs with NCCL, with the NVSwitch multicast
   kernel (``multimem``) and with the peer-memory kernel (``tools/comm_bench.py``), device time MAX over ranks.
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


def schedule_for(world: int):
    """BASELINE config 2's switching schedule scaled to ``world`` GPUs (SP on whenever TP > 1); ends at TP1."""
    def s(tp, pp=1):
        return dict(world_size=world, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp,
                    sequence_parallel=tp > 1)
    if world >= 8:
        return [s(8), s(4), s(2, 2), s(1)]
    if world == 4:
        return [s(4), s(2), s(2, 2), s(1)]
    if world == 2:
        return [s(2), s(1, 2), s(1)]
    return []


def short(strategy) -> str:
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy

    S = ParallelStrategy.from_any(strategy)
    out = ""
    if S.tensor_model_parallel_size > 1:
        out += f"tp{S.tensor_model_parallel_size}"
    if S.pipeline_model_parallel_size > 1:
        out += f"pp{S.pipeline_model_parallel_size}"
    out += f"dp{S.data_parallel_size}"
    return out + ("-sp" if S.sequence_parallel else "")


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
    ap.add_argument("--reshard-iters", type=int, default=5, help="round trips per switch pair (0: no switching)")
    ap.add_argument("--strategy-steps", type=int, default=2, help="timed steps per strategy of the schedule")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-context", action="store_true", help="skip the other engines' timings")
    ap.add_argument("--no-allreduce", action="store_true", help="skip the all-reduce comparison (phase 6)")
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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    from elasticmegatron_b200.config import Args, TrainConfig, preset, set_args
    from elasticmegatron_b200.ops.native import ext, launch_count
    from elasticmegatron_b200.parallel.process_groups import ProcessGroupPool, create_all_groups
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
                     train_iters=1000, overlap_grad_reduce=world > 1, overlap_param_gather=world > 1, seed=0)
    set_args(Args(model=cfg, train=tc))
    tp, pp = args.tp, args.pp
    base = dict(world_size=world, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp,
                sequence_parallel=tp > 1)
    S = ParallelStrategy(**base)
    par = short(base)
    sched = schedule_for(world) if (world > 1 and args.reshard_iters > 0) else []
    strategies = [base] + [s for s in sched if ParallelStrategy(**s) != S]
    if world > 1:
        create_all_groups([ParallelStrategy(**s) for s in strategies])
    ts = TrainingState(S)
    ts.init_weights(0, method="local")
    it = DataloaderState.build_iterators(ts, 0)[0]
    tokens_per_step = gbs * cfg.seq_length

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def timed_steps(state, itr, n):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            train_step(state, itr, return_loss=False)
        e1.record()
        barrier()
        return e0.elapsed_time(e1)

    for _ in range(args.warmup):
        train_step(ts, it, return_loss=False)
    barrier()
    samples, stop = [], threading.Event()
    th = threading.Thread(target=_clock_sampler, args=(local, stop, samples), daemon=True)
    th.start()
    time.sleep(0.3)
    n0 = launch_count()
    ms = timed_steps(ts, it, args.steps)
    launches = launch_count() - n0
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
    ms, e2e_ms_max, launches = max_over_ranks([ms, e2e_ms or 0.0, float(launches)])
    value = tokens_per_step * args.steps / (ms / 1e3)

    per_strategy, switches, context, link_gbs, checksum_ok = None, None, None, None, None
    if sched:
        try:
            per_strategy, switches, context, link_gbs, checksum_ok = switching_phases(
                args, world, strategies, sched, ts, tokens_per_step, timed_steps, barrier, max_over_ranks)
        except Exception as e:  # report, never lose the throughput line
            per_strategy = {"error": repr(e)[:400]}
    allreduce = None
    if world > 1 and not args.no_allreduce:
        try:
            from elasticmegatron_b200.tools.comm_bench import run as allreduce_bench

            allreduce = allreduce_bench(dist.group.WORLD, [256], iters=10, warmup=3)
        except Exception as e:
            allreduce = {"error": repr(e)[:400]}
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
            # GEMM calls that ran on the library because the tcgen05 kernels could not take their operands
            "gemm_fallbacks": int(getattr(ext(), "gemm_fallback_count", lambda: -1)()),
            "strategies": per_strategy,
            "switches": switches,
            "link_gbs_measured": link_gbs,
            "link_gbs_nominal": 900.0,
            "checksum_ok": checksum_ok,
            "context_engines": context,
            "allreduce_256mb": allreduce,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def switching_phases(args, world, strategies, sched, ts, tokens_per_step, timed_steps, barrier, max_over_ranks):
    """Phases 3-5 of the module docstring (every rank runs the same collectives in the same order)."""
    import torch

    from elasticmegatron_b200.parallel.process_groups import ProcessGroupPool
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.transfer.validate import state_checksum
    from elasticmegatron_b200.utils.links import measure_peer_copy_gbs

    # the NVLink kernel engine on GPUs; host ranks (the CPU plumbing test of these phases) use batched P2P
    mgr = ElasticMegatronManager(strategies, training_state=ts,
                                 engine="native" if torch.cuda.is_available() else "torch")
    world_g = ProcessGroupPool.get(list(range(world)))
    # 3. tokens/s per strategy of the schedule
    per = []
    for s in sched:
        st = mgr.reshard(s)
        itr = mgr.build_iterators(0)[0]
        make_room_for_activations()
        train_step_untimed(st, itr)
        ms = max_over_ranks([timed_steps(st, itr, args.strategy_steps)])[0]
        per.append({"strategy": short(s), "tokens_per_s": tokens_per_step * args.strategy_steps / (ms / 1e3),
                    "ms_per_step": ms / args.strategy_steps, "steps": args.strategy_steps})
    # 4. switch latency per consecutive pair (schedule is a cycle: it ends at the base layout)
    link = measure_peer_copy_gbs() if torch.cuda.is_available() else None
    chain = [sched[-1]] + sched
    switches, all_ok = [], True
    for a, b in zip(chain[:-1], chain[1:]):
        if ParallelStrategy(**a) == ParallelStrategy(**b):
            continue
        st = mgr.reshard(a)
        ref = state_checksum(st, world_g)
        lat = {"fwd": [], "back": []}
        ok = True
        rec = {}
        for i in range(2 * args.reshard_iters):
            dst = b if i % 2 == 0 else a
            st = mgr.reshard(dst)
            sw = mgr.last_switch
            lat["fwd" if i % 2 == 0 else "back"].append(sw["transfer_ms"])
            if i % 2 == 0 and not rec:
                rec = dict(sw)
            if i < 2 or i == 2 * args.reshard_iters - 1:
                ok &= state_checksum(st, world_g) == ref
        all_ok &= ok
        p50f, p50b = statistics.median(lat["fwd"]), statistics.median(lat["back"])
        roof = rec.get("nvlink_roofline_ms") or 0.0
        roof_m = rec.get("nvlink_roofline_ms_measured") or 0.0
        switches.append({"src": short(a), "dst": short(b), "p50_ms": p50f, "p50_ms_back": p50b,
                         "all_ms": lat["fwd"], "all_ms_back": lat["back"], "gbytes": rec.get("gbytes"),
                         "roofline_ms_900": roof, "roofline_frac_900": roof / p50f if p50f else None,
                         "roofline_ms_measured": roof_m, "roofline_frac_measured": roof_m / p50f if p50f else None,
                         "total_ms_first": rec.get("total_ms"), "checksum_ok": bool(ok)})
    # 5. other engines of this repository on the first pair (context, not the reference)
    context = None
    if not args.no_context:
        context = {"note": "repo code: batched NCCL P2P engine and a re-implementation of the reference's transfer "
                           "schedule on this framework's layouts; not the reference's own build"}
        a, b = sched[-1], sched[0]
        mgr.reshard(a)
        native_engine, native_name = mgr.engine, mgr.engine_name
        for name in ("torch", "reference"):
            mgr.engine, mgr.engine_name = mgr._make_engine(name), name
            mgr.reshard(b)
            context[name] = {"src": short(a), "dst": short(b), "transfer_ms": mgr.last_switch["transfer_ms"]}
            mgr.engine, mgr.engine_name = native_engine, native_name
            mgr.reshard(a)
    barrier()
    return per, switches, context, link, bool(all_ok)


def make_room_for_activations(min_free_frac: float = 0.25) -> None:
    """Before training under a new layout: when less than ``min_free_frac`` of the GPU is free, return the arena
    pool's cached (released) state arenas to the driver.  The cache keeps up to 40 % of the device for fast
    switch-backs; with 2 GPUs a 7B state plus a full cache plus a step's activations comes close to the device's
    size.  Local to each rank (no collective)."""
    import torch

    if not torch.cuda.is_available():
        return
    free, total = torch.cuda.mem_get_info()
    if free < min_free_frac * total:
        from elasticmegatron_b200.runtime.memory import get_pool

        get_pool(torch.device("cuda", torch.cuda.current_device())).trim()


def train_step_untimed(st, itr):
    from elasticmegatron_b200.runtime.train import train_step

    train_step(st, itr, return_loss=False)


if __name__ == "__main__":
    main()
