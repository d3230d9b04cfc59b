"""Data parallelism over flat, bucketed parameter / gradient arenas.

Behaviour matched to what the reference drives in Megatron's DDP (elastic_megatron/megatron_manager/
training_state.py:109-137, 176-197, 199-311): one contiguous param buffer and one fp32 gradient buffer per
rank, bucketed; gradients are reduce-scattered (ZeRO-1) bucket by bucket, optionally overlapped with
backward, then all-reduced across Group-ZeRO instances; after the optimizer step the parameter buckets
are all-gathered.  The layout comes from ``planner/layout.py`` so the reshard planner sees exactly the
buffers used here.

On CUDA the bucket collectives are this framework's kernels: the reduce-scatter and the parameter all-gather
pull over NVLink peer memory (``dp_comm.py``, ``EMB_DP_PEER=0`` for NCCL), and the Group-ZeRO cross-instance
all-reduce goes through NVSwitch multicast or peer memory (``nvls.py``, ``EMB_NVLS=0`` for NCCL).

Gradient scaling: buckets are reduced with SUM and the optimizer scales the own shard by ``1/(DP*CP)``
(dense and expert alike: expert replicas jointly see the tokens of every DP*CP rank).  Parameters whose
gradients are partial sums across TP ranks under sequence parallelism (norm weights, router) are first
all-reduced over the TP group.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..planner.layout import RankLayout
from . import dp_comm, nvls


def _rs_inplace(buf: torch.Tensor, shard_index: int, group, async_op: bool = False):
    """Reduce-scatter (SUM) ``buf`` over ``group``; shard ``shard_index`` of ``buf`` receives the result.
    With ``async_op`` the collective runs on the communicator's stream and the returned work is waited later
    (the gradients of the bucket are final, so backward may continue meanwhile)."""
    if group is None:
        return None
    n = dist.get_world_size(group)
    if n == 1:
        return None
    if buf.is_cuda:
        c = buf.numel() // n
        return dist.reduce_scatter_tensor(buf[shard_index * c:(shard_index + 1) * c], buf, group=group,
                                          async_op=async_op)
    return dist.all_reduce(buf, group=group, async_op=async_op)


def _ag_inplace(buf: torch.Tensor, shard_index: int, group, async_op: bool = False):
    if group is None:
        return None
    n = dist.get_world_size(group)
    if n == 1:
        return None
    c = buf.numel() // n
    if buf.is_cuda:
        return dist.all_gather_into_tensor(buf, buf[shard_index * c:(shard_index + 1) * c], group=group,
                                           async_op=async_op)
    parts = list(buf.chunk(n))
    mine = parts[shard_index].clone()
    dist.all_gather(parts, mine, group=group)
    return None


class _EventWait:
    """A CUDA event with the ``wait()`` of a collective's work handle: the current stream waits for it."""

    def __init__(self, ev):
        self.ev = ev

    def wait(self):
        torch.cuda.current_stream().wait_event(self.ev)


def _param_key(lp) -> object:
    """Which part of the forward first reads a parameter: its layer, 'pre' (embedding) or 'post' (final norm,
    output layer)."""
    if lp.layer_local is not None:
        return lp.layer_local
    return "pre" if lp.name.startswith("embedding") else "post"


class DistributedDataParallel:
    def __init__(self, layout: RankLayout, pstate, params: Dict[str, torch.nn.Parameter],
                 param_arena: torch.Tensor, grad_arena: torch.Tensor, overlap_grad_reduce: bool = False):
        self.layout, self.ps = layout, pstate
        self.params = params
        self.overlap = overlap_grad_reduce
        self.param_arena, self.grad_arena = param_arena, grad_arena
        s = pstate.strategy
        self.sp = bool(s.sequence_parallel) and s.tensor_model_parallel_size > 1
        self._hooks = []
        self.peer = None
        self._peer_stale = True
        self.bind(param_arena, grad_arena)
        self._pending: List = []
        self._ready: Dict[int, int] = {}
        self._launched = set()
        self._rs_works: List = []
        # in-flight parameter all-gathers: (forward keys the bucket's parameters belong to, work)
        self._ag_pending: List = []
        self._bucket_keys = {}
        for kind, bl in (("dense", layout.dense), ("expert", layout.expert)):
            if bl is None:
                continue
            for b in range(len(bl.buckets)):
                self._bucket_keys[(kind, b)] = {_param_key(bl.params[j]) for j in bl.bucket_params[b]}
        # gradient reduction is only started from backward hooks while this is True (the last
        # micro-batch); earlier micro-batches just accumulate (the reference's ``no_sync``)
        self.sync_enabled = True
        for p in params.values():
            self._hooks.append(p.register_post_accumulate_grad_hook(self._make_acc_hook(p)))
            p._grad_ready = self._make_ready(p)

    # ------------------------------------------------------------------ memory binding
    def bind(self, param_arena: torch.Tensor, grad_arena: Optional[torch.Tensor]) -> None:
        self.param_arena, self.grad_arena = param_arena, grad_arena
        self._peer_stale = True  # peers map the new arenas at the next step start (a collective point)
        for name, p in self.params.items():
            off = self.layout.offset_by_name[name]
            n = p._local_param.numel
            if grad_arena is not None:
                p.main_grad = grad_arena[off:off + n].view(p._local_param.shape)
            else:
                p.main_grad = None

    def _make_acc_hook(self, p):
        def hook(param):
            if param.grad is not None:
                param.main_grad.add_(param.grad.view(param.main_grad.shape).to(param.main_grad.dtype))
                param.grad = None
                param._grad_ready()
        return hook

    def _make_ready(self, p):
        def ready():
            if not self.overlap or not self.sync_enabled:
                return
            # bucket bookkeeping for overlap: a bucket is reduced once all its params reported
            b = self._bucket_of.get(id(p))
            if b is None:
                return
            self._ready[b] = self._ready.get(b, 0) + 1
            if self._ready[b] == self._bucket_sizes[b]:
                self._launch_bucket(b)
        return ready

    # ------------------------------------------------------------------ grad sync
    def _bucket_views(self):
        """(kind, bucket index, grad view, shard index, zero group, inter group)."""
        out = []
        L = self.layout
        for kind, bl, base, gname, iname, zi in (
                ("dense", L.dense, 0, "zero", "zero_inter", L.dense_shard_index),
                ("expert", L.expert, L.dense.numel, "expert_zero", "expert_zero_inter", L.expert_shard_index)):
            if bl is None:
                continue
            for b, (s, e) in enumerate(bl.buckets):
                out.append((kind, b, base + s, base + e, zi, self.ps.groups.get(gname), self.ps.groups.get(iname)))
        return out

    def _ensure_peer(self) -> None:
        """(Re)build the peer-memory collectives after the arenas changed; collective over the shard groups, so
        it runs at the step start, which every rank of the strategy reaches together."""
        if not self._peer_stale and self.peer is not None and not self.peer.current(self._bucket_views()):
            self._peer_stale = True  # its flag buffer was released or the groups were re-created
        if not self._peer_stale:
            return
        self._peer_stale = False
        self.peer = None
        if (self.grad_arena is None or not self.grad_arena.is_cuda or not dp_comm.enabled()
                or not dist.is_initialized()):
            return
        views = self._bucket_views()
        if not any(g is not None and dist.get_world_size(g) > 1 for _, _, _, _, _, g, _ in views):
            return
        self.peer = dp_comm.PeerDP(views, self.grad_arena, self.param_arena, self.param_arena.element_size())

    def prepare(self):
        """Per-step bucket bookkeeping for overlapped reduction."""
        self._ensure_peer()
        if self.peer is not None:
            self.peer.begin_step()
        self._ready = {}
        self._pending = []
        self._bucket_of = {}
        self._bucket_sizes = {}
        self._launched = set()
        if not self.overlap:
            return
        for i, (kind, b, s, e, zi, g, ig) in enumerate(self._bucket_views()):
            bl = self.layout.dense if kind == "dense" else self.layout.expert
            names = [bl.params[j].name for j in bl.bucket_params[b]]
            ps = [self.params[n] for n in names]
            # SP-partial params need a TP all-reduce first, and tied-embedding copies a sum over the embedding
            # group (and, at PP=1, report ready from both the embedding and the head): keep their buckets for
            # the end of backward
            if self.sp and any(p._local_param.sp_partial for p in ps):
                continue
            if any(p._local_param.tied for p in ps):
                continue
            for p in ps:
                self._bucket_of[id(p)] = i
            self._bucket_sizes[i] = len(ps)

    def _launch_bucket(self, i: int):
        kind, b, s, e, zi, g, ig = self._bucket_views()[i]
        if i in self._launched:
            return
        self._launched.add(i)
        # asynchronous: the reduction of this bucket overlaps the rest of backward
        if self.peer is not None:
            self.peer.reduce_scatter(i)
            return
        w = _rs_inplace(self.grad_arena[s:e], zi, g, async_op=True)
        if w is not None:
            self._rs_works.append(w)

    def zero_grad(self) -> None:
        if self.grad_arena is not None:
            self.grad_arena.zero_()
        self.prepare()

    def finish_grad_sync(self) -> None:
        if self.sp and self.ps.size("tp") > 1:
            parts = [p.main_grad.view(-1) for p in self.params.values() if p._local_param.sp_partial]
            if parts:
                flat = torch.cat(parts)
                dist.all_reduce(flat, group=self.ps.group("tp"))
                o = 0
                for t in parts:
                    t.copy_(flat[o:o + t.numel()])
                    o += t.numel()
        tied = [p for p in self.params.values() if p._local_param.tied]
        eg = self.ps.groups.get("embedding")
        if tied and eg is not None and dist.get_world_size(eg) > 1:
            # the first stage's word embedding and the last stage's output-layer copy of it: one gradient
            # (Megatron's embedding-group all-reduce; the reference moves the pair with transfer.py:103-141)
            for p in tied:
                dist.all_reduce(p.main_grad, group=eg)
        views = self._bucket_views()
        for w in self._rs_works:
            w.wait()
        self._rs_works = []
        for i, (kind, b, s, e, zi, g, ig) in enumerate(views):
            if i not in getattr(self, "_launched", set()):
                if self.peer is not None:
                    self.peer.reduce_scatter(i, side_stream=False)
                else:
                    _rs_inplace(self.grad_arena[s:e], zi, g)
        if self.peer is not None:
            self.peer.wait_reduce_scatters()
            self.wait_params()  # every all-gather pull of the last step read its peers' shards already
            self.peer.end_step()  # nobody overwrites gradients a peer may still read
        # Group-ZeRO: replicas of one shard all-reduce across instances
        for i, (kind, b, s, e, zi, g, ig) in enumerate(views):
            if ig is not None and dist.get_world_size(ig) > 1:
                n = dist.get_world_size(g) if g is not None else 1
                c = (e - s) // n
                # NVSwitch multicast reduction (peer memory without it; NCCL with EMB_NVLS=0)
                nvls.all_reduce_(self.grad_arena[s + zi * c:s + (zi + 1) * c], ig)

    def start_param_sync(self, overlap: bool = False) -> None:
        """All-gather the updated parameter shards, bucket by bucket.  With ``overlap`` the gathers are left in
        flight, launched in the order the next forward needs them (the buffer holds parameters in reverse
        forward order, so the last bucket first); the forward waits for each bucket just before the first layer
        that reads it (``wait_params``), and every other reader of the arena waits for all of them."""
        self.wait_params()
        views = self._bucket_views()
        if self.peer is not None:
            for i, ev in self.peer.all_gather(list(reversed(range(len(views)))), overlap):
                kind, b = views[i][0], views[i][1]
                self._ag_pending.append((self._bucket_keys.get((kind, b), set()), _EventWait(ev)))
            return
        for kind, b, s, e, zi, g, ig in reversed(views):
            if g is None:
                continue
            w = _ag_inplace(self.param_arena[s:e], zi, g, async_op=overlap)
            if w is not None:
                self._ag_pending.append((self._bucket_keys.get((kind, b), set()), w))

    def wait_params(self, key=None) -> None:
        """Make the current stream wait for the in-flight parameter all-gathers of the buckets that hold
        parameters read first by ``key`` (a local layer index, 'pre' or 'post'); all of them when None."""
        if not self._ag_pending:
            return
        keep = []
        for keys, w in self._ag_pending:
            if key is None or key in keys:
                w.wait()
            else:
                keep.append((keys, w))
        self._ag_pending = keep

    def remove_hooks(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
