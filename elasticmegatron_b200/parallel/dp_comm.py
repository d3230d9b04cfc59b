"""Data-parallel bucket collectives over NVLink peer memory (K6 gradient reduce-scatter, K7 parameter all-gather).

The ranks of a ZeRO shard group map each other's gradient and parameter arenas (CUDA IPC, once per arena) and
share a small flag array (a symmetric buffer of the group).  Per bucket:

* ``reduce_scatter(i)``: this rank signals "my gradients of bucket i are final" on the compute stream (a flag
  store into every peer's array), then a pull kernel on the side stream waits for every rank's flag and sums the
  rank's own shard slice from all ranks, in rank order, into its own arena (``csrc/comm/dp_collectives.cu``);
* ``all_gather(i)``: after the optimizer step this rank signals "my parameter shard of bucket i is final"; the
  pull kernel copies every peer's shard of the bucket into this rank's arena.

Both run on a side stream so that backward (reduce-scatter) and the next forward (all-gather) continue; the
caller waits per bucket through the returned events.  ``end_step`` is a barrier over the flag memory after the
step's reduce-scatters: no rank zeroes or overwrites gradients that a peer may still be reading.  Parameter
shards are rewritten only by the next optimizer step, which comes after that barrier of the next step, by when
every rank's forward has waited for its own all-gather pulls.

Epochs increase once per step and are kept on the shared flag buffer, so a new layout's DDP over the same group
never mistakes an old flag for a new one.  ``EMB_DP_PEER=0`` selects the NCCL collectives instead.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..ops.native import ext

MAX_BUCKETS = 512  # per collective kind; flag slots: kind * MAX_BUCKETS + bucket
_TIMEOUT_MS = int(os.environ.get("EMB_DP_PEER_TIMEOUT_MS", "60000"))


def enabled() -> bool:
    return os.environ.get("EMB_DP_PEER", "1") != "0"


def _handle(t: torch.Tensor) -> bytes:
    return bytes(ext().ipc_get_handle(t).numpy().tobytes())


def _open(h: bytes) -> int:
    return int(ext().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))


class _Group:
    """One ZeRO shard group: the peers' arena addresses and the shared flag buffer."""

    def __init__(self, group, grad_arena: torch.Tensor, param_arena: torch.Tensor):
        from ..ops.tp_fused import _buffer

        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        assert self.n <= 8, "peer-memory DP collectives cover one NVSwitch domain (<= 8 ranks)"
        dev = grad_arena.device
        self.buf = _buffer(group, 4096, dev, "dp_flags", 4096)
        if not hasattr(self.buf, "dp_epoch"):
            self.buf.dp_epoch = 0
        self.flags = self.buf.flags  # int64 [n]: flag-array base of every rank (after the barrier signals)
        mine = (_handle(grad_arena), _handle(param_arena))
        allh = [None] * self.n
        dist.all_gather_object(allh, mine, group=group)
        g, p = [], []
        for r, (hg, hp) in enumerate(allh):
            if r == self.me:
                g.append(grad_arena.data_ptr())
                p.append(param_arena.data_ptr())
            else:
                g.append(_open(hg))
                p.append(_open(hp))
        self.grad_ptrs = torch.tensor(g, dtype=torch.int64)
        self.param_ptrs = torch.tensor(p, dtype=torch.int64)


class PeerDP:
    """K6 / K7 for one rank's DDP: ``views`` are the DDP's bucket views (kind, b, start, end, shard index,
    group, inter group) in the DDP's order."""

    def __init__(self, views, grad_arena: torch.Tensor, param_arena: torch.Tensor, param_el: int):
        self.views = views
        self.param_el = param_el
        self.stream = torch.cuda.Stream(device=grad_arena.device)
        self.groups: Dict[int, _Group] = {}
        assert len(views) <= MAX_BUCKETS
        for kind, b, s, e, zi, g, ig in views:
            if g is not None and dist.get_world_size(g) > 1 and id(g) not in self.groups:
                self.groups[id(g)] = _Group(g, grad_arena, param_arena)
        self._rs_events: List[torch.cuda.Event] = []
        self.epoch: Dict[int, int] = {}

    def current(self, views) -> bool:
        """False once a flag buffer was closed (symmetric buffers released) or ``views`` name other groups."""
        if any(G.buf.closed for G in self.groups.values()):
            return False
        return [id(v[5]) for v in views] == [id(v[5]) for v in self.views]

    def begin_step(self) -> None:
        """Advance every group's epoch (all ranks of a group call it once per step)."""
        for k, G in self.groups.items():
            G.buf.dp_epoch += 1
            self.epoch[k] = G.buf.dp_epoch

    def _group(self, i: int) -> Tuple[Optional[_Group], tuple]:
        v = self.views[i]
        g = v[5]
        return (self.groups.get(id(g)) if g is not None else None), v

    def reduce_scatter(self, i: int, side_stream: bool = True) -> None:
        G, (kind, b, s, e, zi, g, ig) = self._group(i)
        if G is None:
            return
        ep = self.epoch[id(g)]
        ext().dp_signal(G.flags, G.me, i, 1, ep)
        c = (e - s) // G.n
        off = (s + G.me * c) * 4
        if side_stream:
            cur = torch.cuda.current_stream()
            self.stream.wait_stream(cur)
            with torch.cuda.stream(self.stream):
                ext().dp_rs_pull(G.grad_ptrs, G.me, off, c, G.flags, i, ep, _TIMEOUT_MS)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self._rs_events.append(ev)
        else:
            ext().dp_rs_pull(G.grad_ptrs, G.me, off, c, G.flags, i, ep, _TIMEOUT_MS)

    def wait_reduce_scatters(self) -> None:
        cur = torch.cuda.current_stream()
        for ev in self._rs_events:
            cur.wait_event(ev)
        self._rs_events = []

    def end_step(self) -> None:
        """Barrier over each group's flag memory: every rank's pulls of this step are done."""
        for G in self.groups.values():
            G.buf.barrier()

    def all_gather(self, order: List[int], overlap: bool) -> List[Tuple[int, torch.cuda.Event]]:
        """Signal every bucket's own shard, then pull the peers' shards bucket by bucket in ``order``; returns
        (view index, event) per launched pull (the current stream already waits when ``overlap`` is False)."""
        kinds = {}
        for i in order:
            G, v = self._group(i)
            if G is not None:
                kinds.setdefault(id(v[5]), (G, []))[1].append(i)
        for G, idx in kinds.values():
            ep = self.epoch[id(G.group)]
            lo, hi = min(idx), max(idx)
            ext().dp_signal(G.flags, G.me, MAX_BUCKETS + lo, hi - lo + 1, ep)
        out = []
        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)
        for i in order:
            G, (kind, b, s, e, zi, g, ig) = self._group(i)
            if G is None:
                continue
            c = (e - s) // G.n
            with torch.cuda.stream(self.stream):
                ext().dp_ag_pull(G.param_ptrs, G.me, s * self.param_el, c * self.param_el, G.flags,
                                 MAX_BUCKETS + i, self.epoch[id(g)], _TIMEOUT_MS)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            out.append((i, ev))
        if not overlap:
            for _, ev in out:
                cur.wait_event(ev)
            out = []
        return out
