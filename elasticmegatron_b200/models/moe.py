"""Mixtral-style MoE layer: softmax top-k router, switch load-balancing loss, EP all-to-all, grouped experts.

Behaviour follows the reference's MoE launch configuration (run_moe.sh:61-68: 8 experts, top-2, aux loss
coefficient 1e-2, all-to-all dispatcher, grouped GEMM).  Routing: ``probs = softmax(topk(logits))``;
aux loss ``= E * coeff / (T^2 * k) * sum_e(sum_t softmax(logits)[t, e] * count_e)`` (Switch Transformer
load balancing).  Experts use ETP = 1: each EP rank holds ``E / EP`` whole experts stacked as
``fc1 [E_loc, 2f, h]`` / ``fc2 [E_loc, h, f]``.
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from ..ops import functional as F_


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_splits: List[int], recv_splits: List[int], group):
        ctx.group, ctx.send, ctx.recv = group, send_splits, recv_splits
        out = torch.empty((sum(recv_splits),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, dy):
        out = torch.empty((sum(ctx.send),) + tuple(dy.shape[1:]), dtype=dy.dtype, device=dy.device)
        dist.all_to_all_single(out, dy.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


def all_to_all(x, send_splits, recv_splits, group):
    if group is None or dist.get_world_size(group) == 1:
        return x
    return _AllToAll.apply(x, send_splits, recv_splits, group)


class GroupedLinearFn(torch.autograd.Function):
    """y[seg_e] = x[seg_e] @ W[e]^T for consecutive token segments; dW[e] accumulates into main_grad[e]."""

    @staticmethod
    def forward(ctx, x, w, counts: List[int]):
        ctx.counts = counts
        ctx.save_for_backward(x, w)
        y = x.new_empty((x.shape[0], w.shape[1]))
        o = 0
        for e, n in enumerate(counts):
            if n:
                F_.gemm(x[o:o + n], w[e], trans_b=True, out=y[o:o + n])
            o += n
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.zeros_like(x)
        mg = getattr(w, "main_grad", None)
        dw = None if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        tgt = mg.view(w.shape) if mg is not None else dw
        o = 0
        for e, n in enumerate(ctx.counts):
            if n:
                F_.gemm(dy[o:o + n], w[e], out=dx[o:o + n])
                F_.gemm(dy[o:o + n], x[o:o + n], trans_a=True, out=tgt[e], accumulate=True)
            o += n
        if mg is not None:
            hook = getattr(w, "_grad_ready", None)
            if hook is not None:
                hook()
            return dx, None, None
        return dx, dw.to(w.dtype), None


class MoELayer:
    def __init__(self, cfg, pstate, w_router, w_fc1, w_fc2):
        self.cfg, self.ps = cfg, pstate
        self.wr, self.w1, self.w2 = w_router, w_fc1, w_fc2
        self.ep = pstate.strategy.expert_model_parallel_size
        self.ep_group = pstate.group("ep") if self.ep > 1 else None
        self.E = cfg.num_experts
        self.E_loc = self.E // self.ep
        self.k = cfg.moe_router_topk
        s = pstate.strategy
        self.sp_group = pstate.group("tp") if (s.tensor_model_parallel_size > 1 and s.sequence_parallel) else None

    def __call__(self, h: torch.Tensor):
        T = h.shape[0]
        E, k, E_loc, ep = self.E, self.k, self.E_loc, self.ep
        logits = F_.linear(h, self.wr).float()
        top_logits, top_idx = logits.topk(k, dim=-1)
        probs = torch.softmax(top_logits, -1)
        scores = torch.softmax(logits, -1)
        counts = torch.bincount(top_idx.reshape(-1), minlength=E)
        # Under sequence parallelism the aux loss is defined over the whole sequence: expert counts are
        # summed over the TP group and each rank contributes its tokens' share of sum_t softmax(logits).
        T_full, counts_full = T, counts
        if self.sp_group is not None:
            counts_full = counts.clone()
            dist.all_reduce(counts_full, group=self.sp_group)
            T_full = T * dist.get_world_size(self.sp_group)
        aux = (E * self.cfg.moe_aux_loss_coeff / (T_full * T_full * k)) * (
            scores.sum(0) * counts_full.to(scores.dtype)).sum()
        flat = top_idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        token_of = order // k
        x_perm = h[token_of]
        cnt = counts.view(ep, E_loc)
        if ep > 1:
            recv = torch.empty_like(cnt)
            dist.all_to_all_single(recv, cnt.contiguous(), group=self.ep_group)
        else:
            recv = cnt
        send_splits = cnt.sum(1).tolist()
        recv_splits = recv.sum(1).tolist()
        x_recv = all_to_all(x_perm, send_splits, recv_splits, self.ep_group)
        # rows arrive grouped by (source rank, local expert); regroup by local expert
        recv_l = recv.tolist()
        src_off, idx = [], []
        o = 0
        for r in range(ep):
            src_off.append(o)
            o += sum(recv_l[r])
        seg_start = {}
        for r in range(ep):
            oo = src_off[r]
            for e in range(E_loc):
                seg_start[(r, e)] = oo
                oo += recv_l[r][e]
        for e in range(E_loc):
            for r in range(ep):
                s0 = seg_start[(r, e)]
                idx.append(torch.arange(s0, s0 + recv_l[r][e], device=h.device))
        perm = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long, device=h.device)
        ecounts = [sum(recv_l[r][e] for r in range(ep)) for e in range(E_loc)]
        xe = x_recv[perm]
        a = GroupedLinearFn.apply(xe, self.w1, ecounts)
        a = F_.swiglu(a)
        ye = GroupedLinearFn.apply(a, self.w2, ecounts)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=h.device)
        y_recv = ye[inv]
        y_perm = all_to_all(y_recv, recv_splits, send_splits, self.ep_group)
        wts = probs.reshape(-1)[order].to(y_perm.dtype)
        out = torch.zeros_like(h).index_add(0, token_of, y_perm * wts[:, None])
        return out, aux
