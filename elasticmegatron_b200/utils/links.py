"""NVLink bandwidth used for the roofline of transfers: the nominal figure and one measured in the job.

NVLink 5 gives each B200 18 links, 900 GB/s per direction through the NVSwitch to any peer.  The figure a copy
can actually reach is measured with the transfer engine's own kernel (K1, ``reshard_copy``): every rank pushes
``nbytes`` from a local buffer into the next rank's buffer (mapped through CUDA IPC), all ranks at once, and
the device time (CUDA events, MAX over ranks) gives the per-direction rate.  Switch records report the
roofline at both rates; ``EMB_NVLINK_GBS`` overrides the measured one.
"""
from __future__ import annotations

import os
from typing import Optional

NVLINK_NOMINAL_GBS = 900.0
_measured: Optional[float] = None


def measured_link_gbs() -> Optional[float]:
    e = os.environ.get("EMB_NVLINK_GBS")
    if e:
        return float(e)
    return _measured


def set_measured_link_gbs(v: Optional[float]) -> None:
    global _measured
    _measured = v


def measure_peer_copy_gbs(nbytes: int = 1 << 30, iters: int = 5, group=None) -> float:
    """Per-direction peer-copy bandwidth (GB/s) of the K1 kernel, every rank writing to rank + 1 at once.
    Collective over ``group`` (default: the world); records the result for later switch reports."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from ..ops.native import ext
    from ..transfer.native_engine import TASK_DTYPE

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    dev = torch.cuda.current_device()
    src = ext().arena_alloc(nbytes, dev)
    dst = ext().arena_alloc(nbytes, dev)
    src.fill_(1)
    h = bytes(ext().ipc_get_handle(dst).numpy().tobytes())
    hs = [None] * world
    dist.all_gather_object(hs, h, group=group)
    peer = (rank + 1) % world
    paddr = int(ext().ipc_open(torch.frombuffer(bytearray(hs[peer]), dtype=torch.uint8)))
    chunk = 8 << 20
    n = nbytes // chunk
    t = np.zeros(n, dtype=TASK_DTYPE)
    t["src"] = src.data_ptr() + np.arange(n, dtype=np.uint64) * chunk
    t["dst"] = paddr + np.arange(n, dtype=np.uint64) * chunk
    t["rows"] = 1
    t["row_bytes"] = chunk
    t["planes"] = 1
    t["flags"] = 1
    buf = torch.from_numpy(t.view(np.uint8).copy()).cuda()
    flag = torch.zeros(1, device="cuda")
    ms = []
    for i in range(iters + 1):
        dist.all_reduce(flag, group=group)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ext().reshard_copy(buf, n, 0)
        e1.record()
        torch.cuda.synchronize()
        if i:
            ms.append(e0.elapsed_time(e1))
    dist.all_reduce(flag, group=group)
    torch.cuda.synchronize()
    ext().ipc_close(torch.frombuffer(bytearray(hs[peer]), dtype=torch.uint8))
    v = torch.tensor([sorted(ms)[len(ms) // 2]], device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX, group=group)
    gbs = nbytes / (float(v.item()) / 1e3) / 1e9
    del src, dst
    set_measured_link_gbs(gbs)
    return gbs
