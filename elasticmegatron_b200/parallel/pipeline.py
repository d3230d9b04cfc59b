"""Forward/backward schedules: no pipelining (gradient accumulation) and non-interleaved 1F1B.

Pipeline activations travel with ``torch.distributed`` batched isend/irecv (NCCL on GPUs, Gloo on CPU) over
the PP group, as Megatron's schedules do for the reference (forward_backward_func, external; no virtual
pipeline stages, reference README:197).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


class AttachAux(torch.autograd.Function):
    """Return ``x`` unchanged; in backward, feed gradient ``scale`` into the scalar ``aux`` loss."""

    @staticmethod
    def forward(ctx, x, aux, scale):
        ctx.scale = scale
        ctx.dtype, ctx.device = aux.dtype, aux.device
        return x.view_as(x)

    @staticmethod
    def backward(ctx, dy):
        return dy, torch.full((), ctx.scale, dtype=ctx.dtype, device=ctx.device), None


class StepContext:
    """What a schedule needs from the model side for one optimizer step."""

    def __init__(self, stage, pstate, ddp, num_microbatches: int, act_shape: Tuple[int, ...], act_dtype,
                 device, loss_scale: float, get_batch: Callable[[int], Tuple]):
        self.stage, self.ps, self.ddp = stage, pstate, ddp
        self.num_mb = num_microbatches
        self.act_shape, self.act_dtype, self.device = act_shape, act_dtype, device
        self.loss_scale = loss_scale  # multiplies sum(token losses) of one micro-batch
        self.get_batch = get_batch
        self.loss_sums: List[torch.Tensor] = []


def _fwd(ctx: StepContext, mb: int, inp: Optional[torch.Tensor]):
    ids, labels = ctx.get_batch(mb)
    ps = ctx.ps
    x = ids if ps.is_first_stage else inp
    out, aux = ctx.stage(x, labels if ps.is_last_stage else None)
    if ps.is_last_stage:
        s = out.sum()
        ctx.loss_sums.append(s.detach())
        loss = s * ctx.loss_scale
        if aux is not None:
            loss = loss + aux / ctx.num_mb
        return loss
    if aux is not None:
        out = AttachAux.apply(out, aux, 1.0 / ctx.num_mb)
    return out


def _bwd(ctx: StepContext, inp, out, dout):
    if inp is not None:
        inp.retain_grad()
    if dout is None:
        torch.autograd.backward(out)
    else:
        torch.autograd.backward(out, dout)
    return inp.grad if inp is not None else None


def _p2p(ops):
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()


def forward_backward_no_pipelining(ctx: StepContext):
    for mb in range(ctx.num_mb):
        ctx.ddp.sync_enabled = mb == ctx.num_mb - 1
        loss = _fwd(ctx, mb, None)
        _bwd(ctx, None, loss, None)
    ctx.ddp.sync_enabled = True
    return ctx.loss_sums


def forward_backward_1f1b(ctx: StepContext):
    ps = ctx.ps
    pp, rank = ps.pp_size, ps.pp_rank
    g = ps.group("pp")
    warm = min(pp - rank - 1, ctx.num_mb)
    rem = ctx.num_mb - warm
    inputs, outputs = [], []
    shape, dt, dev = ctx.act_shape, ctx.act_dtype, ctx.device

    def recv_fwd():
        if ps.is_first_stage:
            return None
        t = torch.empty(shape, dtype=dt, device=dev, requires_grad=True)
        _p2p([dist.P2POp(dist.irecv, t, ps.prev_rank, g)])
        return t

    def send_fwd(y):
        if not ps.is_last_stage:
            _p2p([dist.P2POp(dist.isend, y.detach().contiguous(), ps.next_rank, g)])

    def send_fwd_recv_bwd(y):
        if ps.is_last_stage:
            return None
        dy = torch.empty(shape, dtype=dt, device=dev)
        _p2p([dist.P2POp(dist.isend, y.detach().contiguous(), ps.next_rank, g),
              dist.P2POp(dist.irecv, dy, ps.next_rank, g)])
        return dy

    def send_bwd(dx):
        if not ps.is_first_stage:
            _p2p([dist.P2POp(dist.isend, dx.contiguous(), ps.prev_rank, g)])

    def send_bwd_recv_fwd(dx):
        if ps.is_first_stage:
            return None
        t = torch.empty(shape, dtype=dt, device=dev, requires_grad=True)
        _p2p([dist.P2POp(dist.isend, dx.contiguous(), ps.prev_rank, g),
              dist.P2POp(dist.irecv, t, ps.prev_rank, g)])
        return t

    def recv_bwd():
        if ps.is_last_stage:
            return None
        dy = torch.empty(shape, dtype=dt, device=dev)
        _p2p([dist.P2POp(dist.irecv, dy, ps.next_rank, g)])
        return dy

    mb_f = 0
    mb_b = 0
    ctx.ddp.sync_enabled = False
    for _ in range(warm):
        x = recv_fwd()
        y = _fwd(ctx, mb_f, x)
        mb_f += 1
        send_fwd(y)
        inputs.append(x)
        outputs.append(y)
    x = recv_fwd() if rem > 0 else None
    for i in range(rem):
        y = _fwd(ctx, mb_f, x)
        mb_f += 1
        dy = send_fwd_recv_bwd(y)
        inputs.append(x)
        outputs.append(y)
        xi, yi = inputs.pop(0), outputs.pop(0)
        ctx.ddp.sync_enabled = mb_b == ctx.num_mb - 1
        dx = _bwd(ctx, xi, yi, dy)
        mb_b += 1
        if i == rem - 1:
            x = None
            send_bwd(dx)
        else:
            x = send_bwd_recv_fwd(dx)
    for _ in range(warm):
        xi, yi = inputs.pop(0), outputs.pop(0)
        dy = recv_bwd()
        ctx.ddp.sync_enabled = mb_b == ctx.num_mb - 1
        dx = _bwd(ctx, xi, yi, dy)
        mb_b += 1
        send_bwd(dx)
    ctx.ddp.sync_enabled = True
    return ctx.loss_sums


def get_forward_backward_func(pp_size: int):
    return forward_backward_1f1b if pp_size > 1 else forward_backward_no_pipelining
