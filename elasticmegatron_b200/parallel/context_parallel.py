"""Context parallelism: attention over a sequence split into 2*CP load-balanced chunks.

CP rank ``r`` holds chunks ``r`` and ``2*CP-1-r`` (so every rank does the same amount of causal work).  Three
ways to exchange keys and values over the CP group (Megatron's ``--cp-comm-type``):

* ``"all_gather"`` (default, :func:`cp_attention`): K and V are all-gathered (reduce-scattered in backward);
  each query chunk is one fused attention call over the global prefix of keys that ends with its own chunk.
* ``"p2p"`` (:func:`cp_ring_attention`): a ring.  Every step each rank sends the K/V block it holds to the
  next CP rank and receives one from the previous; the transfer of step ``t+1`` is posted before the math of
  step ``t``, so the exchange overlaps the attention.  Partial outputs are merged by their log-sum-exp; the
  backward pass sends the K/V blocks round again with their dK/dV accumulators, which end at their owners.
  No rank ever holds more than two K/V blocks.
* ``"a2a"`` (:func:`cp_ulysses_attention`, DeepSpeed-Ulysses): an all-to-all trades the sequence split for a
  split of the query groups, so each rank holds the WHOLE sequence of ``G / CP`` query groups (with their
  K/V heads), runs one fused causal attention over it, and a second all-to-all trades back.  Needs the local
  query-group count divisible by CP; moves 2 x (q + k + v + out) / CP of the activations per rank instead of
  all of K/V.

On CUDA (bf16, head dim 128, chunks a multiple of 128 rows) every variant runs on the native flash-attention
kernels (``csrc/attn``): the all-gather and ring variants as one kernel call per (query chunk, key chunk) block -
the diagonal block causal, earlier chunks in full - whose partial outputs are merged by their log-sum-exp in
fp32 (``attn_merge``); the backward calls the native backward kernel per block with the final output and
log-sum-exp, so every block's probabilities are the global softmax's.  Ulysses runs one native causal call over
the whole sequence.  Elsewhere (CPU, other shapes) the blocks are fp32 tensor algebra / library attention.

In the reference CP lives entirely in Megatron/TE (context_parallel_size is only carried and folded into the
ZeRO group, parallel_strategy.py:131-147).
"""
from __future__ import annotations

import math
from typing import List, Tuple

import torch
import torch.distributed as dist

from ..ops import functional as F_

CP_COMM_TYPES = ("all_gather", "p2p", "a2a")


def _global_chunk_starts(s: int, cp: int):
    """Row offset, inside the rank-ordered all-gather of K/V, of every global chunk 0 .. 2*CP-1."""
    c = s // 2
    out = []
    for g in range(2 * cp):
        r, half = (g, 0) if g < cp else (2 * cp - 1 - g, 1)
        out.append(r * s + half * c)
    return out


def _native_blocks(qkv: torch.Tensor) -> bool:
    """Whether the per-block math runs on the native flash-attention kernels."""
    return (qkv.is_cuda and qkv.dtype == torch.bfloat16 and qkv.shape[-1] == 128 and (qkv.shape[0] // 2) % 128 == 0
            and F_._has_native_attention())


class _Blocks:
    """Attention of this rank's two query chunks against one key / value chunk at a time on the native kernels.

    Each query chunk has a fused ``[c, b, G, hpg + 2, d]`` buffer (the kernels' input layout) whose query slots are
    filled once; a block copies its key / value chunk into the other slots and runs one kernel call."""

    def __init__(self, qkv: torch.Tensor, hpg: int):
        from ..ops.native import ext

        self.ext = ext()
        s, b, G, w, d = qkv.shape
        self.c, self.b, self.G, self.hpg, self.H, self.d = s // 2, b, G, hpg, G * hpg, d
        c = self.c
        self.buf = [torch.empty(c, b, G, w, d, dtype=qkv.dtype, device=qkv.device) for _ in range(2)]
        for h in range(2):
            self.buf[h][:, :, :, :hpg].copy_(qkv[h * c:(h + 1) * c, :, :, :hpg])

    def _load(self, hq: int, kv_chunk: torch.Tensor) -> torch.Tensor:
        self.buf[hq][:, :, :, self.hpg:].copy_(kv_chunk)
        return self.buf[hq]

    def start(self):
        """Fresh accumulators: fp32 outputs [c, b, H, d] and log-sum-exps [b, H, c] (-inf) per query chunk."""
        dev = self.buf[0].device
        out = [torch.empty(self.c, self.b, self.H, self.d, dtype=torch.float32, device=dev) for _ in range(2)]
        lse = [torch.full((self.b, self.H, self.c), float("-inf"), dtype=torch.float32, device=dev)
               for _ in range(2)]
        return out, lse

    def forward(self, hq: int, kv_chunk: torch.Tensor, causal: bool, out, lse) -> None:
        o_b, l_b = self.ext.attn_fwd(self._load(hq, kv_chunk), self.hpg, causal)
        self.ext.attn_merge(out[hq], lse[hq], o_b, l_b)

    def backward(self, hq: int, kv_chunk: torch.Tensor, causal: bool, dout_h, o_h, lse_h, dq, dkv_chunk) -> None:
        """dq[hq] ([c, b, G, hpg, d] fp32) and dkv_chunk ([c, b, G, 2, d] fp32) += this block's gradients."""
        g = self.ext.attn_bwd(dout_h, self._load(hq, kv_chunk), o_h, lse_h, self.hpg, causal)
        dq[hq] += g[:, :, :, :self.hpg]
        dkv_chunk += g[:, :, :, self.hpg:]

    @staticmethod
    def finish(out, dtype) -> torch.Tensor:
        """The two chunks' merged outputs as [s, b, H * d] in ``dtype``."""
        c, b, H, d = out[0].shape
        return torch.cat([o.view(c, b, H * d) for o in out], 0).to(dtype)


def _assemble_dqkv(qkv, hpg, dq, dkv):
    c = qkv.shape[0] // 2
    dqkv = torch.empty_like(qkv)
    for h in range(2):
        dqkv[h * c:(h + 1) * c, :, :, :hpg] = dq[h]
    dqkv[:, :, :, hpg:] = dkv
    return dqkv


class _AGNativeFn(torch.autograd.Function):
    """All-gather CP on the native kernels: K/V gathered in forward, their gradients reduce-scattered back."""

    @staticmethod
    def _gather(qkv, hpg, group, cp):
        s, b, G, _, d = qkv.shape
        kv = qkv[:, :, :, hpg:].contiguous()
        kv_all = torch.empty(cp * s, b, G, 2, d, dtype=kv.dtype, device=kv.device)
        dist.all_gather_into_tensor(kv_all, kv, group=group)
        return kv_all

    @staticmethod
    def forward(ctx, qkv, hpg, group, cp_rank, cp):
        s = qkv.shape[0]
        c = s // 2
        kv_all = _AGNativeFn._gather(qkv, hpg, group, cp)
        starts = _global_chunk_starts(s, cp)
        blk = _Blocks(qkv, hpg)
        out, lse = blk.start()
        for hq, ci in enumerate(_chunks_of(cp_rank, cp)):
            for kj in range(ci + 1):
                blk.forward(hq, kv_all[starts[kj]:starts[kj] + c], kj == ci, out, lse)
        o = _Blocks.finish(out, qkv.dtype)
        ctx.save_for_backward(qkv, o, *lse)
        ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp = hpg, group, cp_rank, cp
        return o

    @staticmethod
    def backward(ctx, dout):
        qkv, o, l0, l1 = ctx.saved_tensors
        hpg, group, cp_rank, cp = ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp
        s, b, G, _, d = qkv.shape
        c = s // 2
        kv_all = _AGNativeFn._gather(qkv, hpg, group, cp)
        starts = _global_chunk_starts(s, cp)
        blk = _Blocks(qkv, hpg)
        dout = dout.contiguous()
        dq = [torch.zeros(c, b, G, hpg, d, dtype=torch.float32, device=qkv.device) for _ in range(2)]
        dkv_all = torch.zeros(cp * s, b, G, 2, d, dtype=torch.float32, device=qkv.device)
        for hq, ci in enumerate(_chunks_of(cp_rank, cp)):
            dout_h, o_h, l_h = dout[hq * c:(hq + 1) * c], o[hq * c:(hq + 1) * c], (l0, l1)[hq]
            for kj in range(ci + 1):
                st = starts[kj]
                blk.backward(hq, kv_all[st:st + c], kj == ci, dout_h, o_h, l_h, dq, dkv_all[st:st + c])
        dkv = torch.empty(s, b, G, 2, d, dtype=torch.float32, device=qkv.device)
        dist.reduce_scatter_tensor(dkv, dkv_all, group=group)  # every rank's contribution to my chunks
        return _assemble_dqkv(qkv, hpg, dq, dkv), None, None, None, None


def cp_attention(qkv: torch.Tensor, hpg: int, group, cp_rank: int, cp: int) -> torch.Tensor:
    """Causal attention of this rank's two query chunks against the gathered keys / values.

    K / V are all-gathered in rank order and re-ordered into global sequence order; query chunk ``ci`` then
    attends to the global prefix ``[0, (ci + 1) * c)`` with a causal mask aligned to the lower right (its
    own chunk is the last block of that prefix), so each chunk is one fused attention call with no explicit
    mask tensor and no K/V head replication (grouped-query attention is native to the call)."""
    from torch.nn.attention.bias import causal_lower_right

    if _native_blocks(qkv):
        return _AGNativeFn.apply(qkv, hpg, group, cp_rank, cp)
    s, b, G, _, d = qkv.shape
    c = s // 2
    kv = qkv[:, :, :, hpg:].contiguous()  # [s, b, G, 2, d]
    kv_all = F_.gather_from_sp(kv.view(s, -1), group).view(cp * s, b, G, 2, d)
    kv_glob = torch.cat([kv_all[st:st + c] for st in _global_chunk_starts(s, cp)], 0)  # global order
    outs = []
    for half, ci in ((0, cp_rank), (1, 2 * cp - 1 - cp_rank)):
        L = (ci + 1) * c
        q = qkv[half * c:(half + 1) * c, :, :, :hpg].reshape(c, b, G * hpg, d).permute(1, 2, 0, 3)
        k = kv_glob[:L, :, :, 0].permute(1, 2, 0, 3)
        v = kv_glob[:L, :, :, 1].permute(1, 2, 0, 3)
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=causal_lower_right(c, L),
                                                             enable_gqa=hpg > 1)
        outs.append(o.permute(2, 0, 1, 3).reshape(c, b, G * hpg * d))
    return torch.cat(outs, 0)


# ------------------------------------------------------------------------------------------------ ring
def _chunks_of(rank: int, cp: int) -> Tuple[int, int]:
    """Global chunk indices held by CP rank ``rank`` (first and second half of its local sequence)."""
    return rank, 2 * cp - 1 - rank


def _relation(qi: int, kj: int) -> int:
    """0: key chunk entirely after the query chunk (skipped); 1: the same chunk (causal); 2: entirely before."""
    return 0 if kj > qi else (1 if kj == qi else 2)


def _scores(q, k, scale, causal):
    """q [b, G, hpg, c, d], k [b, G, c, d] -> fp32 scores [b, G, hpg, c, c] (upper triangle -inf if causal)."""
    s = torch.einsum("bghid,bgjd->bghij", q.float(), k.float()) * scale
    if causal:
        c = s.shape[-1]
        s = s.masked_fill(torch.ones(c, c, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    return s


class _Ring:
    """Posts the exchange of one step's blocks with the CP neighbours (send to next, receive from previous)."""

    def __init__(self, group, cp_rank: int, cp: int):
        ranks = dist.get_process_group_ranks(group)
        self.group, self.nxt, self.prv = group, ranks[(cp_rank + 1) % cp], ranks[(cp_rank - 1) % cp]

    def start(self, send: torch.Tensor) -> Tuple[torch.Tensor, list]:
        send = send.contiguous()
        recv = torch.empty(send.shape, dtype=send.dtype, device=send.device)
        ops = [dist.P2POp(dist.isend, send, self.nxt, self.group), dist.P2POp(dist.irecv, recv, self.prv, self.group)]
        return recv, dist.batch_isend_irecv(ops)

    @staticmethod
    def wait(reqs) -> None:
        for r in reqs:
            r.wait()


def _split_q(qkv: torch.Tensor, hpg: int) -> List[torch.Tensor]:
    """[s, b, G, hpg+2, d] -> the two query chunks as [b, G, hpg, c, d]."""
    s = qkv.shape[0]
    c = s // 2
    return [qkv[h * c:(h + 1) * c, :, :, :hpg].permute(1, 2, 3, 0, 4) for h in range(2)]


def _split_kv(kv: torch.Tensor) -> List[Tuple[torch.Tensor, torch.Tensor]]:
    """[s, b, G, 2, d] -> ((k, v) of each half) as [b, G, c, d]."""
    c = kv.shape[0] // 2
    return [(kv[h * c:(h + 1) * c, :, :, 0].permute(1, 2, 0, 3), kv[h * c:(h + 1) * c, :, :, 1].permute(1, 2, 0, 3))
            for h in range(2)]


class _RingNativeFn(torch.autograd.Function):
    """The ring on the native kernels: same exchange as :class:`_RingAttnFn`, one kernel call per block."""

    @staticmethod
    def forward(ctx, qkv, hpg, group, cp_rank, cp):
        s = qkv.shape[0]
        c = s // 2
        my = _chunks_of(cp_rank, cp)
        ring = _Ring(group, cp_rank, cp)
        kv = qkv[:, :, :, hpg:].contiguous()
        blk = _Blocks(qkv, hpg)
        out, lse = blk.start()
        for t in range(cp):
            if t + 1 < cp:
                nxt, reqs = ring.start(kv)
            src = (cp_rank - t) % cp
            for hk in range(2):
                kj = _chunks_of(src, cp)[hk]
                for hq in range(2):
                    rel = _relation(my[hq], kj)
                    if rel:
                        blk.forward(hq, kv[hk * c:(hk + 1) * c], rel == 1, out, lse)
            if t + 1 < cp:
                _Ring.wait(reqs)
                kv = nxt
        o = _Blocks.finish(out, qkv.dtype)
        ctx.save_for_backward(qkv, o, *lse)
        ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp = hpg, group, cp_rank, cp
        return o

    @staticmethod
    def backward(ctx, dout):
        qkv, o, l0, l1 = ctx.saved_tensors
        hpg, group, cp_rank, cp = ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp
        s, b, G, _, d = qkv.shape
        c = s // 2
        my = _chunks_of(cp_rank, cp)
        ring = _Ring(group, cp_rank, cp)
        blk = _Blocks(qkv, hpg)
        dout = dout.contiguous()
        dq = [torch.zeros(c, b, G, hpg, d, dtype=torch.float32, device=qkv.device) for _ in range(2)]
        kv = qkv[:, :, :, hpg:].contiguous()
        incoming = None
        for t in range(cp):
            if t + 1 < cp:
                nxt_kv, reqs_kv = ring.start(kv)
            src = (cp_rank - t) % cp
            acc = torch.zeros(kv.shape, dtype=torch.float32, device=qkv.device)
            for hk in range(2):
                kj = _chunks_of(src, cp)[hk]
                for hq in range(2):
                    rel = _relation(my[hq], kj)
                    if rel:
                        blk.backward(hq, kv[hk * c:(hk + 1) * c], rel == 1, dout[hq * c:(hq + 1) * c],
                                     o[hq * c:(hq + 1) * c], (l0, l1)[hq], dq, acc[hk * c:(hk + 1) * c])
            if incoming is not None:
                _Ring.wait(incoming[1])
                acc += incoming[0]
            incoming = ring.start(acc)
            if t + 1 < cp:
                _Ring.wait(reqs_kv)
                kv = nxt_kv
        _Ring.wait(incoming[1])
        return _assemble_dqkv(qkv, hpg, dq, incoming[0]), None, None, None, None


class _RingAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, hpg, group, cp_rank, cp):
        s, b, G, _, d = qkv.shape
        c = s // 2
        scale = 1.0 / math.sqrt(d)
        qs = _split_q(qkv, hpg)
        my = _chunks_of(cp_rank, cp)
        ring = _Ring(group, cp_rank, cp)
        kv = qkv[:, :, :, hpg:].contiguous()
        out = [torch.zeros(b, G, hpg, c, d, dtype=torch.float32, device=qkv.device) for _ in range(2)]
        lse = [torch.full((b, G, hpg, c), float("-inf"), dtype=torch.float32, device=qkv.device) for _ in range(2)]
        for t in range(cp):
            if t + 1 < cp:
                nxt, reqs = ring.start(kv)
            src = (cp_rank - t) % cp
            for hk, (k, v) in enumerate(_split_kv(kv)):
                kj = _chunks_of(src, cp)[hk]
                for hq in range(2):
                    rel = _relation(my[hq], kj)
                    if rel == 0:
                        continue
                    sc = _scores(qs[hq], k, scale, rel == 1)
                    l_b = torch.logsumexp(sc, -1)
                    o_b = torch.einsum("bghij,bgjd->bghid", torch.exp(sc - l_b[..., None]), v.float())
                    l_n = torch.logaddexp(lse[hq], l_b)
                    out[hq] = out[hq] * torch.exp(lse[hq] - l_n)[..., None] + o_b * torch.exp(l_b - l_n)[..., None]
                    lse[hq] = l_n
            if t + 1 < cp:
                _Ring.wait(reqs)
                kv = nxt
        ctx.save_for_backward(qkv, *out, *lse)
        ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp = hpg, group, cp_rank, cp
        o = torch.cat([x.permute(3, 0, 1, 2, 4).reshape(c, b, G * hpg * d) for x in out], 0)
        return o.to(qkv.dtype)

    @staticmethod
    def backward(ctx, dout):
        qkv, o0, o1, l0, l1 = ctx.saved_tensors
        hpg, group, cp_rank, cp = ctx.hpg, ctx.group, ctx.cp_rank, ctx.cp
        s, b, G, _, d = qkv.shape
        c = s // 2
        scale = 1.0 / math.sqrt(d)
        qs = _split_q(qkv, hpg)
        my = _chunks_of(cp_rank, cp)
        ring = _Ring(group, cp_rank, cp)
        dos = [dout[h * c:(h + 1) * c].reshape(c, b, G, hpg, d).permute(1, 2, 3, 0, 4).float() for h in range(2)]
        outs, lses = (o0, o1), (l0, l1)
        D = [(dos[h] * outs[h]).sum(-1) for h in range(2)]  # [b, G, hpg, c]
        dq = [torch.zeros(b, G, hpg, c, d, dtype=torch.float32, device=qkv.device) for _ in range(2)]
        # the block in flight: K/V of rank src, and the fp32 dK/dV ([s, b, G, 2, d]) accumulated for it by the
        # ranks it has visited, which arrives one step behind it; after CP hops the sum is back at src
        kv = qkv[:, :, :, hpg:].contiguous()
        incoming = None
        for t in range(cp):
            if t + 1 < cp:
                nxt_kv, reqs_kv = ring.start(kv)
            src = (cp_rank - t) % cp
            acc = torch.zeros(kv.shape, dtype=torch.float32, device=qkv.device)
            for hk, (k, v) in enumerate(_split_kv(kv)):
                kj = _chunks_of(src, cp)[hk]
                dk = acc[hk * c:(hk + 1) * c, :, :, 0].permute(1, 2, 0, 3)
                dv = acc[hk * c:(hk + 1) * c, :, :, 1].permute(1, 2, 0, 3)
                for hq in range(2):
                    rel = _relation(my[hq], kj)
                    if rel == 0:
                        continue
                    p = torch.exp(_scores(qs[hq], k, scale, rel == 1) - lses[hq][..., None])  # [b, G, hpg, c, c]
                    dv += torch.einsum("bghij,bghid->bgjd", p, dos[hq])
                    dp = torch.einsum("bghid,bgjd->bghij", dos[hq], v.float())
                    ds = p * (dp - D[hq][..., None]) * scale
                    dq[hq] += torch.einsum("bghij,bgjd->bghid", ds, k.float())
                    dk += torch.einsum("bghij,bghid->bgjd", ds, qs[hq].float())
            if incoming is not None:
                _Ring.wait(incoming[1])
                acc += incoming[0]
            incoming = ring.start(acc)
            if t + 1 < cp:
                _Ring.wait(reqs_kv)
                kv = nxt_kv
        _Ring.wait(incoming[1])
        dkv = incoming[0]
        dqkv = torch.empty_like(qkv)
        for h in range(2):
            dqkv[h * c:(h + 1) * c, :, :, :hpg] = dq[h].permute(3, 0, 1, 2, 4).to(qkv.dtype)
        dqkv[:, :, :, hpg:] = dkv.to(qkv.dtype)
        return dqkv, None, None, None, None


def cp_ring_attention(qkv: torch.Tensor, hpg: int, group, cp_rank: int, cp: int) -> torch.Tensor:
    """Causal attention of this rank's two query chunks with K/V passed round the CP ring.

    Same inputs and output as :func:`cp_attention` (``qkv`` [s, b, G, hpg+2, d] after RoPE, out
    [s, b, G*hpg*d]).  Scores, softmax statistics and accumulators are fp32 whatever the input dtype; the
    math is plain tensor algebra, so the same code runs on the host and on the device; on CUDA it runs on the native
    kernels (:class:`_RingNativeFn`)."""
    if _native_blocks(qkv):
        return _RingNativeFn.apply(qkv, hpg, group, cp_rank, cp)
    return _RingAttnFn.apply(qkv, hpg, group, cp_rank, cp)


# --------------------------------------------------------------------------------------------- ulysses
class _AllToAll(torch.autograd.Function):
    """Equal-split all-to-all over dim 0 (``[CP, ...]``: slot j goes to CP rank j, slot i comes from rank i).
    Its adjoint is the same exchange, so the backward pass is one more all-to-all of the gradient.  Both
    buffers are dense: the incoming gradient is often a permuted view, and a receive buffer shaped after it
    with ``empty_like`` would keep its strides while the collective writes contiguous bytes."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _AllToAll._exchange(x, group)

    @staticmethod
    def backward(ctx, dy):
        return _AllToAll._exchange(dy, ctx.group), None

    @staticmethod
    def _exchange(x, group):
        x = x.contiguous()
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x, group=group)
        return out


def cp_ulysses_attention(qkv: torch.Tensor, hpg: int, group, cp_rank: int, cp: int) -> torch.Tensor:
    """Causal attention with the CP split moved from the sequence to the query groups and back.

    Same inputs and output as :func:`cp_attention`.  Query group slice ``j`` (``G / CP`` groups) of every
    rank's two chunks goes to rank ``j``; rank ``j`` puts the ``2 * CP`` chunks in global order, attends over
    the whole sequence with one fused causal call (grouped-query attention native to it) and sends each rank
    its own two chunks back."""
    s, b, G, w, d = qkv.shape
    if G % cp:
        raise ValueError(f"cp_comm_type a2a needs the local query groups ({G}) divisible by CP ({cp})")
    gp, c, S = G // cp, s // 2, cp * s
    x = qkv.reshape(s, b, cp, gp, w, d).permute(2, 0, 1, 3, 4, 5)  # [dest rank, s, b, gp, hpg+2, d]
    y = _AllToAll.apply(x.contiguous(), group)  # [source rank, s, b, gp, hpg+2, d]
    chunks = [y[g, :c] if g < cp else y[2 * cp - 1 - g, c:] for g in range(2 * cp)]
    full = torch.cat(chunks, 0)  # [S, b, gp, hpg+2, d], global sequence order
    if full.is_cuda:
        # the gathered sequence is already the fused layout of the attention op (native kernels on CUDA)
        o = F_.attention(full.contiguous(), hpg).view(S, b, gp, hpg * d)
    else:
        q = full[:, :, :, :hpg].reshape(S, b, gp * hpg, d).permute(1, 2, 0, 3)
        k = full[:, :, :, hpg].permute(1, 2, 0, 3)
        v = full[:, :, :, hpg + 1].permute(1, 2, 0, 3)
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=hpg > 1)
        o = o.permute(2, 0, 1, 3).reshape(S, b, gp, hpg * d)
    back = torch.stack([torch.cat([o[j * c:(j + 1) * c], o[(2 * cp - 1 - j) * c:(2 * cp - j) * c]], 0)
                        for j in range(cp)])  # [dest rank, s, b, gp, hpg*d]
    r = _AllToAll.apply(back, group)  # [query group slice, s, b, gp, hpg*d]
    return r.permute(1, 2, 0, 3, 4).reshape(s, b, G * hpg * d)
