"""Inter-process elastic training: a running job hands its state to a NEW job with another size and layout.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 --master-port 29500 \
        examples/inter_process/train_handoff.py --model llama2-7b --strategy ws8 \
        --successor-strategy ws4-tp2 --successor-nproc 4 --handoff-at 5 --train-iters 20

``--chain a,b,c`` runs several hops (e.g. 8 -> 4 -> 8 GPUs with Group-ZeRO replicas dropped and rebuilt); every
job behaves as below towards the next one.

Old job ("primary"): trains on ``--strategy``; at iteration ``--handoff-at`` its rank 0 starts the successor
job (``torchrun`` with ``--successor-nproc`` ranks on ``--successor-port``) through ``runtime/agent.py``, then
keeps training and checks once per iteration whether the successor is ready (built its process group and
model).  When it is, every old rank publishes its state in place (``export_state``: CUDA-IPC handles of the
parameter and optimizer arenas, or shared memory on CPU, plus LR / scheduler / data position), waits until
every successor rank has acknowledged, and exits.

Successor: builds the new layout, maps the old processes' arenas and pulls exactly its new shards out of them
(one K1 copy launch on GPUs; ``runtime/interprocess.py``), acknowledges, and continues training from the next
iteration with the same data stream.

This is the analogue of the reference's inter-process example (examples/inter_process/training_011.py:
check_reshard :103-119, role dispatch :414-432, loop hook :1538-1552) and its agent
(tools/agent/env_utils.py:214-483).  ``--cpu`` runs it on gloo ranks.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys
import tempfile
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))  # run from a checkout


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seq-length", type=int, default=None)
    ap.add_argument("--chain", default=None,
                    help="comma list of strategies, one job each, e.g. ws8-inst2,ws4,ws8-inst2 (8 -> 4 -> 8 GPUs); "
                         "job h hands off at iteration (h + 1) * --handoff-at (overrides --strategy / "
                         "--successor-strategy)")
    ap.add_argument("--strategy", default="ws2")
    ap.add_argument("--successor-strategy", default="ws1")
    ap.add_argument("--successor-nproc", type=int, default=None, help="default: world size of the successor")
    ap.add_argument("--successor-port", type=int, default=29700)
    ap.add_argument("--handoff-at", type=int, default=3)
    ap.add_argument("--block-at-handoff", action="store_true",
                    help="wait for the successor at --handoff-at instead of training on until it is ready")
    ap.add_argument("--wait-successor", action="store_true", help="old rank 0 waits for the successor to finish")
    ap.add_argument("--handoff-root", default=None)
    ap.add_argument("--train-iters", type=int, default=8)
    ap.add_argument("--micro-batch-size", type=int, default=1)
    ap.add_argument("--global-batch-size", type=int, default=8)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--timeout", type=float, default=600.0)
    ap.add_argument("--cpu", action="store_true")
    return ap.parse_args(argv)


def _log(rank, it, n, loss, ms, strategy, tag):
    if rank == 0:
        print(f" iteration {it:8d}/{n:8d} | elapsed time per iteration (ms): {ms:.1f} | lm loss: {loss:.6E}"
              f" | strategy: {strategy} | job: {tag}", flush=True)


def main(argv=None):
    a = parse_args(argv)
    from elasticmegatron_b200.config import Args, TrainConfig, get_args, preset, set_args
    from elasticmegatron_b200.parallel.process_groups import ProcessGroupPool, create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime import agent
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import ack, adopt, export_state, import_records, wait_for_acks
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and not a.cpu
    if use_cuda:
        torch.cuda.set_device(local)
    dist.init_process_group("nccl" if use_cuda else "gloo", timeout=datetime.timedelta(seconds=600),
                            **({"device_id": torch.device("cuda", local)} if use_cuda else {}))
    over = {"max_tensor_parallel_size": 8}
    if a.layers:
        over["num_layers"] = a.layers
    if a.seq_length:
        over["seq_length"] = a.seq_length
    over["params_dtype"] = "bf16" if use_cuda else "fp32"  # the CUDA kernels are bf16; CPU ranks run fp32
    set_args(Args(model=preset(a.model, **over),
                  train=TrainConfig(micro_batch_size=a.micro_batch_size, global_batch_size=a.global_batch_size,
                                    lr=a.lr, train_iters=a.train_iters)))
    args = get_args()
    # the jobs of the run: hop h trains under chain[h] and hands its state to hop h + 1
    chain = [ParallelStrategy.parse(x) for x in (a.chain.split(",") if a.chain else
                                                    [a.strategy, a.successor_strategy])]
    hop = int(os.environ.get("EMB_HOP", "0"))
    me_s = chain[hop]
    nxt = chain[hop + 1] if hop + 1 < len(chain) else None
    last_iter = a.handoff_at * (hop + 1) if nxt is not None else None  # iteration at which the next job starts
    gloo_world = ProcessGroupPool.get(list(range(world)), "gloo")
    create_all_groups([me_s])
    ts = TrainingState(me_s) if rank < me_s.world_size else None
    tag_me = f"hop{hop}"
    if hop == 0:
        if ts is not None:
            ts.init_weights(a.seed)
        start = 1
        root = a.handoff_root or (tempfile.mkdtemp(prefix="emb_handoff_") if rank == 0 else None)
        obj = [root]
        dist.broadcast_object_list(obj, src=0, group=gloo_world)
        root = obj[0]
    else:
        root, _ = agent.handoff_location()
        agent.mark_ready(root, tag_me, rank)
        recs = import_records(root, tag_me, old_world=chain[hop - 1].world_size, timeout=a.timeout)
        info = adopt(ts, recs) if ts is not None else None
        ack(root, tag_me, rank)
        start = int(recs[0]["iteration"]) + 1
        args.iteration = start - 1
        args.consumed_train_samples = int(recs[0]["consumed_train_samples"])
        if rank == 0 and info is not None:
            print(f"job {hop} adopted {info['src_strategy']} -> {me_s} at iteration {start - 1}", flush=True)
    it = DataloaderState.build_iterators(ts, args.consumed_train_samples)[0] if ts is not None else None
    job = "primary" if hop == 0 else f"successor{hop}" if len(chain) > 2 else "successor"
    tag_next = f"hop{hop + 1}"
    n_new = (a.successor_nproc if (a.successor_nproc and len(chain) == 2) else nxt.world_size) if nxt else 0
    child, spawned = None, False
    for i in range(start, a.train_iters + 1):
        if spawned and agent.ready_consensus(root, tag_next, n_new, gloo_world):
            break
        if ts is not None:
            t0 = time.perf_counter()
            out = train_step(ts, it)
            _log(rank, i, a.train_iters, out["loss"], (time.perf_counter() - t0) * 1e3, me_s, job)
        args.iteration = i
        args.consumed_train_samples += a.global_batch_size
        if nxt is not None and i == last_iter:
            if rank == 0:
                script = os.path.abspath(__file__)
                cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n_new}",
                       "--master-addr=127.0.0.1", f"--master-port={a.successor_port + hop}", script] + \
                    (argv if argv is not None else sys.argv[1:])
                child = agent.spawn_successor(cmd, root, tag_next, env={"EMB_HOP": str(hop + 1)},
                                              log_path=os.path.join(root, f"{tag_next}.log"))
            spawned = True
            if a.block_at_handoff:
                if rank == 0:
                    agent.wait_ready(root, tag_next, n_new, timeout=a.timeout)
                dist.barrier(group=gloo_world)
    if nxt is not None:
        if ts is not None:
            export_state(ts, root, tag_next)
            wait_for_acks(root, tag_next, n_new, timeout=a.timeout)
        dist.barrier(group=gloo_world)
        if rank == 0:
            print(f"job {hop} exported {me_s} at iteration {args.iteration}; next job's log: "
                  f"{os.path.join(root, tag_next + '.log')}", flush=True)
            if a.wait_successor and child is not None:
                rc = child.wait(timeout=a.timeout)
                with open(os.path.join(root, f"{tag_next}.log")) as f:
                    sys.stdout.write(f.read())
                print(f"successor exit code {rc}", flush=True)
    else:
        dist.barrier(group=gloo_world)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
