"""Inter-process mode: hand a running job's state to a new job with a different topology, in place.

Reference behaviour (elastic_megatron/transfer/ipc_manager.py:54-245, tools/agent/env_utils.py:214-483): the
old job exports each optimizer tensor as a CUDA-IPC handle and sends the handles plus rng / iteration /
scheduler state in one pickled ZeroMQ message per local device, then destroys its process group and exits
right away (which races the consumer's clone); the new job maps the handles and clones the tensors into a
meta-built model, then runs an ordinary reshard.

Here:

* each old rank publishes one record (arena handles, strategy, optimizer / scheduler state, data position)
  through a rendezvous directory - written to a temp file and renamed, so readers never see partial records;
* each new rank maps every old rank's arenas (CUDA IPC on GPUs; shared-memory tensors on CPU) and pulls its
  *new* layout straight out of the old processes' memory - the plan goes from the old strategy to the new
  one and on GPUs it runs in one K1 launch over the mapped addresses; there is no intermediate copy of the
  old layout;
* the old processes keep their arenas alive until every new rank has acknowledged (bounded wait), fixing the
  exporter-exits-too-early hazard.

All waits are bounded by ``timeout`` seconds and raise ``TimeoutError``.
"""
from __future__ import annotations

import io
import os
import pickle
import time
from typing import Dict, List, Optional

import numpy as np
import torch

from ..config import get_args
from ..parallel.strategy import ParallelStrategy
from ..planner.plan import KIND_OPT, build_plan


def _atomic_write(path: str, data: bytes) -> None:
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def _share_cpu(t: torch.Tensor) -> bytes:
    """Serialize a CPU tensor so another process maps the same memory (file-system shared memory)."""
    from multiprocessing.reduction import ForkingPickler

    import torch.multiprocessing  # registers torch's tensor reductions with ForkingPickler

    torch.multiprocessing.set_sharing_strategy("file_system")
    t.share_memory_()
    buf = io.BytesIO()
    ForkingPickler(buf, pickle.HIGHEST_PROTOCOL).dump(t)
    return buf.getvalue()


def export_state(ts, root: str, tag: str, extra: Optional[Dict] = None) -> str:
    """Publish this rank's state for a successor job; the arenas stay valid while ``ts`` is alive."""
    args = get_args()
    d = os.path.join(root, tag)
    os.makedirs(d, exist_ok=True)
    rec = {
        "rank": ts.rank, "pid": os.getpid(), "strategy": ts.strategy.to_dict(),
        "param_numel": ts.layout.param_numel, "opt_numel": ts.layout.opt_numel,
        "param_dtype": str(ts.param_dtype), "device": str(ts.device),
        "optimizer": ts.optimizer.state_dict(), "scheduler": ts.opt_param_scheduler.state_dict(),
        "iteration": args.iteration, "consumed_train_samples": args.consumed_train_samples,
        "extra": extra or {},
    }
    if ts.device.type == "cuda":
        from ..ops.native import ext

        rec["param_handle"] = bytes(ext().ipc_get_handle(ts.param_flat).numpy().tobytes())
        rec["opt_handle"] = bytes(ext().ipc_get_handle(ts.opt_flat).numpy().tobytes())
        rec["device_index"] = ts.device.index
    else:
        rec["param_shared"] = _share_cpu(ts.param_flat)
        rec["opt_shared"] = _share_cpu(ts.opt_flat)
    path = os.path.join(d, f"export_{ts.rank}.pkl")
    _atomic_write(path, pickle.dumps(rec))
    return path


def wait_for_acks(root: str, tag: str, n: int, timeout: float = 600.0) -> None:
    """Old ranks: block until ``n`` successor ranks have acknowledged (they no longer read our memory)."""
    d = os.path.join(root, tag)
    t0 = time.time()
    while True:
        acks = [f for f in os.listdir(d) if f.startswith("ack_")] if os.path.isdir(d) else []
        if len(acks) >= n:
            return
        if time.time() - t0 > timeout:
            raise TimeoutError(f"only {len(acks)} of {n} successor ranks acknowledged within {timeout}s")
        time.sleep(0.05)


def ack(root: str, tag: str, rank: int) -> None:
    _atomic_write(os.path.join(root, tag, f"ack_{rank}"), b"1")


def import_records(root: str, tag: str, old_world: Optional[int] = None, timeout: float = 600.0) -> List[Dict]:
    """New ranks: wait for every old rank's record (bounded) and return them ordered by old rank."""
    d = os.path.join(root, tag)
    t0 = time.time()
    while True:
        recs = {}
        if os.path.isdir(d):
            for f in os.listdir(d):
                if f.startswith("export_") and f.endswith(".pkl"):
                    with open(os.path.join(d, f), "rb") as fh:
                        r = pickle.load(fh)
                    recs[r["rank"]] = r
        if recs:
            ws = old_world or ParallelStrategy(**next(iter(recs.values()))["strategy"]).world_size
            if len(recs) >= ws:
                return [recs[i] for i in range(ws)]
        if time.time() - t0 > timeout:
            raise TimeoutError(f"old job published {len(recs)} records within {timeout}s")
        time.sleep(0.05)


def _map_cpu(blob: bytes) -> torch.Tensor:
    torch.multiprocessing.set_sharing_strategy("file_system")
    return pickle.loads(blob)


def adopt(ts, records: List[Dict]) -> Dict:
    """Fill ``ts`` (the new layout on this rank) from the old job's memory; returns the misc state applied."""
    args = get_args()
    cfg, tc = args.model, args.train
    src = ParallelStrategy.from_any(records[0]["strategy"])
    plan = build_plan(src, ts.strategy, cfg, overlap_grad_reduce=tc.overlap_grad_reduce,
                      ddp_bucket_size=tc.ddp_bucket_size)
    me = ts.rank
    if ts.device.type == "cuda":
        from ..ops.native import ext
        from ..transfer.native_engine import NativeP2PEngine

        addrs = {}
        for r, rec in enumerate(records):
            p = int(ext().ipc_open(torch.frombuffer(bytearray(rec["param_handle"]), dtype=torch.uint8)))
            o = int(ext().ipc_open(torch.frombuffer(bytearray(rec["opt_handle"]), dtype=torch.uint8)))
            addrs[r] = (p, o, 0, 0)
        mine = addrs.get(me, (0, 0, 0, 0))
        addrs[me] = (mine[0], mine[1], ts.param_flat.data_ptr(), ts.opt_flat.data_ptr())
        eng = NativeP2PEngine(mode="pull")
        tasks = eng._tasks(plan, me, addrs, ts.param_flat.element_size())
        if len(tasks):
            buf = torch.from_numpy(tasks.view(np.uint8).copy()).to(ts.device)
            ext().reshard_copy(buf, len(tasks), 0)
        torch.cuda.synchronize(ts.device)
    else:
        from ..transfer.torch_engine import _opt_view, _view

        sp = {r: _map_cpu(rec["param_shared"]) for r, rec in enumerate(records)}
        so = {r: _map_cpu(rec["opt_shared"]) for r, rec in enumerate(records)}
        d = plan.desc
        for row in d[d["dst_rank"] == me]:
            s, R, C = int(row["src_rank"]), int(row["rows"]), int(row["cols"])
            if row["kind"] == KIND_OPT:
                _opt_view(ts.opt_flat, int(row["dst_off"]), R, C, int(row["dst_stride"])).copy_(
                    _opt_view(so[s], int(row["src_off"]), R, C, int(row["src_stride"])))
            else:
                _view(ts.param_flat, int(row["dst_off"]), R, C, int(row["dst_stride"])).copy_(
                    _view(sp[s], int(row["src_off"]), R, C, int(row["src_stride"])))
    rec0 = records[0]
    ts.optimizer.load_state_dict(rec0["optimizer"])
    ts.opt_param_scheduler.load_state_dict(rec0["scheduler"])
    args.iteration = rec0["iteration"]
    args.consumed_train_samples = rec0["consumed_train_samples"]
    return {"iteration": rec0["iteration"], "consumed_train_samples": rec0["consumed_train_samples"],
            "src_strategy": src}
