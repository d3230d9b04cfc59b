"""Expert-parallel MoE dispatch and combine over NVLink peer memory.

Replaces "local re-layout, NCCL all-to-all, local re-layout" on both sides of the expert MLP.  After the
router, the ranks of the expert-parallel group exchange their per-expert assignment counts (one small NCCL
all-gather, read on the host: the sizes of the next tensors depend on them).  From the counts every rank knows
every rank's expert-grouped input layout (per local expert, segments padded to the grouped GEMM's 128-row tile),
so:

* dispatch - one kernel stores each assignment's token row straight into the owning rank's landing buffer at
  its final row of that layout, together with an origin entry (source rank, assignment index); one peer-flag
  barrier; the receiver zero-fills its segment padding and the grouped GEMM consumes the rows as they are;
* combine - one kernel sends every expert output row home to (origin rank, assignment index); one barrier;
  the source sums each token's k rows weighted by the router probabilities.

The backward passes are the same two movements in the other direction (combine backward pushes the weighted
output gradients like a dispatch; dispatch backward returns the input gradients like a combine).

Buffers are symmetric arenas of the EP group (``ops/tp_fused.SymmetricBuffer``) with two halves used on
alternate calls, so a call never overwrites data a peer may still read (each call ends with a barrier that
every rank passes only after finishing its previous calls).  A plan looks its buffers up at every movement: a
later layer with more rows grows (replaces) a buffer, and the plan of an earlier layer, kept for its backward,
must not use the replaced buffer's closed peer mappings.  Every rank of the group asks for the same sizes in the
same order (the sizes are maxima over the group), so a grow stays collective.  Reference behaviour being replaced: Megatron's
alltoall token dispatcher (``--moe-token-dispatcher-type alltoall``, run_moe.sh:66).
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from .native import ext
from .tp_fused import _buffer

SEG_ALIGN = 128


def enabled() -> bool:
    return os.environ.get("EMB_EP_PEER", "1") != "0"


def host_layout(all_counts: np.ndarray, me: int, e_loc: int):
    """From every rank's per-expert assignment counts ``all_counts[src, expert]`` (experts numbered globally,
    expert e living on rank e // e_loc): this rank's segment starts ``seg_me [e_loc + 1]`` and row counts
    ``tot_me [e_loc]``, the first row this rank writes in each global expert's segment ``base [E]`` (rows of
    lower source ranks come first), the expert of each 128-row tile ``tiles``, this rank's layout size and the
    largest over ranks."""
    ep = all_counts.shape[0]
    tot = all_counts.sum(0).reshape(ep, e_loc)  # rows each rank's local experts receive
    pad = (tot + SEG_ALIGN - 1) // SEG_ALIGN * SEG_ALIGN
    seg = np.zeros((ep, e_loc + 1), dtype=np.int64)
    seg[:, 1:] = np.cumsum(pad, 1)
    base = seg[:, :-1].reshape(-1) + all_counts[:me].sum(0)
    seg_me = seg[me]
    cap = int(seg_me[-1])
    tiles = np.full(cap // SEG_ALIGN, -1, dtype=np.int64)
    for e in range(e_loc):
        tiles[seg_me[e] // SEG_ALIGN:seg_me[e + 1] // SEG_ALIGN] = e
    return seg_me, tot[me], base, tiles, cap, int(seg[:, -1].max())


class EPPlan:
    """Where every row of one MoE layer call goes; built collectively by all ranks of the EP group."""

    def __init__(self, group, top: torch.Tensor, counts: torch.Tensor, e_loc: int, hidden: int):
        dev = top.device
        self.group = group
        self.ep = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.T, self.k = top.shape
        self.H = hidden
        E = counts.numel()
        allc = torch.empty(self.ep, E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allc, counts.to(torch.int32).contiguous(), group=group)
        ac = allc.cpu().numpy().astype(np.int64)  # host sync: the next allocations depend on the counts
        seg_me, tot_me, base, tiles, self.cap, self.cap_max = host_layout(ac, self.me, e_loc)
        host = torch.from_numpy(np.concatenate([seg_me, tot_me, base, tiles]).astype(np.int32))
        dv = host.pin_memory().to(dev, non_blocking=True)
        o = 0
        self.seg = dv[o:o + e_loc + 1]; o += e_loc + 1
        self.counts = dv[o:o + e_loc]; o += e_loc
        base_d = dv[o:o + E]; o += E
        self.tiles = dv[o:]
        self.base = base_d
        self.e_loc = e_loc
        self.gid = top.reshape(-1).to(torch.int32).contiguous()
        self.pos_send, self.seg_send, _ = ext().moe_layout(self.gid, counts.to(torch.int32).contiguous(),
                                                           max(self.gid.numel(), 1), 1)
        self.ident = torch.arange(self.T * self.k, device=dev, dtype=torch.int32)
        self.dev = dev
        self.origin = None

    @property
    def land(self):
        return _buffer(self.group, self.cap_max * self.H * 2, self.dev, "ep_land", 1 << 20)

    @property
    def org(self):
        return _buffer(self.group, self.cap_max * 4, self.dev, "ep_org", 1 << 16)

    @property
    def ret(self):
        return _buffer(self.group, self.T * self.k * self.H * 2, self.dev, "ep_ret", 1 << 20)

    def layout(self) -> dict:
        return {"seg": self.seg, "tiles": self.tiles, "counts": self.counts, "cap": self.cap}

    # -------------------------------------------------------------- the four movements
    def push(self, rows: torch.Tensor, w=None, with_origin: bool = False) -> torch.Tensor:
        """rows [T, H] (assignment r uses row r // k, scaled by w[r]) -> this rank's landing rows [cap, H]."""
        lb = self.land
        h = lb.next_half()
        optrs = None
        if with_origin:
            ob = self.org
            ho = ob.next_half()
            optrs = ob.peers[ho]
        ext().ep_push(rows.contiguous(), self.k, self.gid, self.pos_send, self.seg_send, self.base, self.e_loc,
                      None if w is None else w.reshape(-1).float().contiguous(), lb.peers[h], optrs, self.me)
        lb.barrier()
        land = lb.view(h, torch.bfloat16, self.cap_max * self.H)[:self.cap * self.H].view(self.cap, self.H)
        if with_origin:
            org = ob.view(ho, torch.int32, self.cap_max)[:self.cap]
            ext().ep_pad(land, self.seg, self.counts, org)
            self.origin = org.clone()
        else:
            ext().ep_pad(land, self.seg, self.counts, None)
        return land.clone()

    def send_home(self, rows: torch.Tensor) -> torch.Tensor:
        """Landing-layout rows [cap, H] -> this rank's return rows [T * k, H] (its own assignments)."""
        rb = self.ret
        lb = self.land
        h = rb.next_half()
        ext().ep_return(rows.contiguous(), self.origin, self.cap, rb.peers[h])
        lb.barrier()
        n = self.T * self.k
        return rb.view(h, torch.bfloat16, n * self.H).view(n, self.H).clone()


class _EPDispatchFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, plan: EPPlan):
        ctx.plan = plan
        return plan.push(h, None, with_origin=True)

    @staticmethod
    def backward(ctx, dxe):
        plan = ctx.plan
        ret = plan.send_home(dxe)
        return ext().moe_gather(ret, plan.ident, None, plan.T, plan.k), None


class _EPCombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ye, probs, plan: EPPlan):
        ctx.plan = plan
        y_home = plan.send_home(ye)
        pf = probs.reshape(-1).float().contiguous()
        ctx.save_for_backward(y_home, pf)
        return ext().moe_gather(y_home, plan.ident, pf, plan.T, plan.k)

    @staticmethod
    def backward(ctx, dout):
        plan = ctx.plan
        y_home, pf = ctx.saved_tensors
        dout = dout.contiguous()
        dye = plan.push(dout, pf, with_origin=False)
        dprobs = ext().moe_row_dot(dout, plan.k, y_home, plan.ident).view(plan.T, plan.k)
        return dye, dprobs, None


def dispatch(h: torch.Tensor, plan: EPPlan) -> torch.Tensor:
    return _EPDispatchFn.apply(h, plan)


def combine(ye: torch.Tensor, probs: torch.Tensor, plan: EPPlan) -> torch.Tensor:
    return _EPCombineFn.apply(ye, probs, plan)
