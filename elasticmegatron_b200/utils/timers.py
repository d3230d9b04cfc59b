"""Timing utilities.

The reference times a switch with a host wall clock bracketed by ``torch.cuda.synchronize``
(elastic_megatron/resharding/util.py:19-46) and all-reduces MAX over the union group
(elastic_megatron/elastic_manager.py:158-178).  Here the primary clock is CUDA events on the launching
stream (device time); the host clock remains for CPU/gloo runs.  Both report milliseconds and are
reduced with MAX over ranks by :func:`max_over_ranks`.
"""
from __future__ import annotations

import time
from typing import Optional, Sequence

import torch
import torch.distributed as dist


class HostTimer:
    """Wall-clock timer; synchronizes the current CUDA device on both ends when one is in use."""

    def __init__(self, sync: bool = True):
        self.sync = sync and torch.cuda.is_available()
        self.elapsed = 0.0

    def __enter__(self):
        if self.sync:
            torch.cuda.synchronize()
        self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.sync:
            torch.cuda.synchronize()
        self.elapsed = (time.perf_counter() - self._t0) * 1e3
        return False


class DeviceTimer:
    """CUDA-event timer on the current stream (falls back to :class:`HostTimer` on CPU)."""

    def __init__(self, stream: Optional[torch.cuda.Stream] = None):
        self.cuda = torch.cuda.is_available()
        self.stream = stream
        self.elapsed = 0.0

    def __enter__(self):
        if not self.cuda:
            self._host = HostTimer(sync=False).__enter__()
            return self
        s = self.stream or torch.cuda.current_stream()
        self._e0 = torch.cuda.Event(enable_timing=True)
        self._e1 = torch.cuda.Event(enable_timing=True)
        self._e0.record(s)
        return self

    def __exit__(self, *exc):
        if not self.cuda:
            self._host.__exit__(*exc)
            self.elapsed = self._host.elapsed
            return False
        s = self.stream or torch.cuda.current_stream()
        self._e1.record(s)
        self._e1.synchronize()
        self.elapsed = self._e0.elapsed_time(self._e1)
        return False


def max_over_ranks(values: Sequence[float], group=None) -> list:
    """All-reduce MAX of a small vector of floats over ``group`` (no-op without a process group)."""
    if not (dist.is_available() and dist.is_initialized()):
        return list(values)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(list(values), dtype=torch.float64 if dev.type == "cpu" else torch.float32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()


class nvtx_range:
    """NVTX range around a phase (plan, build, transfer, lr, release) so Nsight-style timelines show the
    switch structure; a no-op without CUDA."""

    def __init__(self, name: str):
        self.name = name
        self.on = torch.cuda.is_available()

    def __enter__(self):
        if self.on:
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if self.on:
            torch.cuda.nvtx.range_pop()
        return False
