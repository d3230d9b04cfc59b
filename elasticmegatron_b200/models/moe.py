"""Mixtral-style MoE layer: softmax top-k router, switch load-balancing loss, EP all-to-all, grouped experts.

Behaviour follows the reference's MoE launch configuration (run_moe.sh:61-68: 8 experts, top-2, aux loss
coefficient 1e-2, all-to-all dispatcher, grouped GEMM).  Routing: ``probs = softmax(topk(logits))``;
aux loss ``= E * coeff / (T^2 * k) * sum_e(sum_t softmax(logits)[t, e] * count_e)`` (Switch Transformer
load balancing).  Experts use ETP = 1: each EP rank holds ``E / EP`` whole experts stacked as
``fc1 [E_loc, 2f, h]`` / ``fc2 [E_loc, h, f]``.
"""
from __future__ import annotations

import os
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


# ------------------------------------------------------------------------------------------ native (CUDA) path
# Router, token layout and expert MLP on the extension's kernels (csrc/moe/moe.cu, grouped tcgen05 GEMM in
# csrc/gemm): no per-expert Python loop and, without expert parallelism, no host synchronisation.

def _ext():
    from ..ops.native import ext

    return ext()


class _RouterFn(torch.autograd.Function):
    """(probs [T, k], score_sum [E], top_idx, counts) from fp32 logits; differentiable in probs and score_sum."""

    @staticmethod
    def forward(ctx, logits, k: int):
        top, probs, counts, part = _ext().moe_router_fwd(logits.contiguous(), k)
        ctx.save_for_backward(logits, top, probs)
        ctx.mark_non_differentiable(top, counts)
        return probs, part.sum(0), top, counts

    @staticmethod
    def backward(ctx, dprobs, dscore, _top, _counts):
        logits, top, probs = ctx.saved_tensors
        dprobs = torch.zeros_like(probs) if dprobs is None else dprobs.float().contiguous()
        dscore = torch.zeros(logits.shape[1], device=logits.device) if dscore is None else dscore.float().contiguous()
        return _ext().moe_router_bwd(logits, top, probs, dprobs, dscore), None


class _ScatterFn(torch.autograd.Function):
    """Rows of ``src`` (row r // k_div for assignment r) into the grouped layout ``lay``."""

    @staticmethod
    def forward(ctx, src, lay, k_div: int):
        ctx.lay, ctx.k_div, ctx.n = lay, k_div, src.shape[0]
        return _ext().moe_scatter(src.contiguous(), k_div, lay["pos"], None, lay["seg"], lay["counts"], lay["cap"])

    @staticmethod
    def backward(ctx, d):
        lay = ctx.lay
        return _ext().moe_gather(d.contiguous(), lay["pos"], None, ctx.n, ctx.k_div), None, None


class _GatherFn(torch.autograd.Function):
    """out[i] = sum_j w[i, j] * y[pos[i * k + j]] (w optional); the inverse movement of ``_ScatterFn``."""

    @staticmethod
    def forward(ctx, y, w, lay, n_out: int, k: int):
        ctx.lay, ctx.n_out, ctx.k = lay, n_out, k
        wf = w.reshape(-1).float().contiguous() if w is not None else None
        ctx.has_w = w is not None
        # y is only needed for the gradient of the weights
        ctx.save_for_backward(y if ctx.has_w else torch.empty(0, device=y.device),
                              wf if ctx.has_w else torch.empty(0, device=y.device))
        return _ext().moe_gather(y.contiguous(), lay["pos"], wf, n_out, k)

    @staticmethod
    def backward(ctx, dout):
        y, wf = ctx.saved_tensors
        lay = ctx.lay
        dout = dout.contiguous()
        dy = _ext().moe_scatter(dout, ctx.k, lay["pos"], wf if ctx.has_w else None, lay["seg"], lay["counts"],
                                lay["cap"])
        dw = _ext().moe_row_dot(dout, ctx.k, y.contiguous(), lay["pos"]).view(ctx.n_out, ctx.k) if ctx.has_w else None
        return dy, dw, None, None, None


class _GroupedLinearNativeFn(torch.autograd.Function):
    """y = x @ W[g]^T per 128-row tile of group g (one grouped tcgen05 launch); W [G, out, in]."""

    @staticmethod
    def forward(ctx, x, w, lay):
        ctx.lay = lay
        ctx.save_for_backward(x, w)
        return _ext().gemm_grouped(x.contiguous(), w.contiguous(), True, lay["tiles"])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        lay = ctx.lay
        dy = dy.contiguous()
        dx = _ext().gemm_grouped(dy, w.contiguous(), False, lay["tiles"])
        mg = getattr(w, "main_grad", None)
        if mg is not None:
            _ext().gemm_grouped_wgrad(dy, x, lay["seg"], mg.view(w.shape), True)
            hook = getattr(w, "_grad_ready", None)
            if hook is not None:
                hook()
            return dx, None, None
        dw = torch.empty(w.shape, dtype=torch.float32, device=w.device)
        _ext().gemm_grouped_wgrad(dy, x, lay["seg"], dw, False)
        return dx, dw.to(w.dtype), None


def _layout(gid: torch.Tensor, counts: torch.Tensor, n_rows: int, align: int) -> dict:
    G = counts.numel()
    cap = n_rows + (G * (align - 1) if align > 1 else 0)
    cap = (cap + 127) // 128 * 128 if align > 1 else max(cap, 1)
    pos, seg, tiles = _ext().moe_layout(gid.to(torch.int32).contiguous(), counts.to(torch.int32).contiguous(), cap,
                                        align)
    return {"pos": pos, "seg": seg, "tiles": tiles, "counts": counts.to(torch.int32).contiguous(), "cap": cap}


def native_moe_enabled() -> bool:
    return os.environ.get("EMB_NATIVE_MOE", "1") != "0"


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
        f2 = self.w1.shape[1]
        if (h.is_cuda and native_moe_enabled() and self.E <= 256 and self.k <= 8 and h.shape[1] % 64 == 0
                and f2 % 64 == 0):
            return self._native_forward(h)
        return self._torch_forward(h)

    def _aux(self, score_sum: torch.Tensor, counts: torch.Tensor, T: int) -> torch.Tensor:
        E, k = self.E, self.k
        T_full, counts_full = T, counts
        if self.sp_group is not None:
            counts_full = counts.clone()
            dist.all_reduce(counts_full, group=self.sp_group)
            T_full = T * dist.get_world_size(self.sp_group)
        return (E * self.cfg.moe_aux_loss_coeff / (T_full * T_full * k)) * (score_sum * counts_full.to(score_sum.dtype)).sum()

    def _native_forward(self, h: torch.Tensor):
        """Router kernel -> expert-grouped layout -> grouped fc1 / SwiGLU / fc2 -> weighted combine.

        Without expert parallelism nothing synchronises with the host: the layout is sized for the worst case
        (every segment padded to 128 rows) and the grouped GEMM skips tiles past the last segment.  With EP the
        token counts are exchanged (one small all-gather read on the host) and the rows move over NVLink peer
        memory straight into the owners' grouped layout (``ops/ep_comm.py``; ``EMB_EP_PEER=0``: NCCL
        all-to-all)."""
        T = h.shape[0]
        E, k, E_loc, ep = self.E, self.k, self.E_loc, self.ep
        logits = F_.linear(h, self.wr).float()
        probs, score_sum, top, counts = _RouterFn.apply(logits, k)
        aux = self._aux(score_sum, counts.to(torch.int64), T)
        gid = top.reshape(-1)
        if ep == 1:
            lay = _layout(gid, counts, T * k, 128)
            xe = _ScatterFn.apply(h, lay, k)
            ye = self._experts(xe, lay)
            return _GatherFn.apply(ye, probs, lay, T, k), aux
        from ..ops import ep_comm

        if ep_comm.enabled():
            # expert parallelism over NVLink peer memory: rows go straight into the owners' grouped layout
            plan = ep_comm.EPPlan(self.ep_group, top, counts, E_loc, h.shape[1])
            xe = ep_comm.dispatch(h, plan)
            ye = self._experts(xe, plan.layout())
            return ep_comm.combine(ye, probs, plan), aux
        # NCCL path: dense send buffer grouped by global expert (= by destination rank, local expert)
        send_lay = _layout(gid, counts, T * k, 1)
        x_send = _ScatterFn.apply(h, send_lay, k)
        cnt = counts.view(ep, E_loc)
        recv = torch.empty_like(cnt)
        dist.all_to_all_single(recv, cnt.contiguous(), group=self.ep_group)
        send_splits = cnt.sum(1).tolist()
        recv_splits = recv.sum(1).tolist()
        x_recv = all_to_all(x_send, send_splits, recv_splits, self.ep_group)
        n_recv = int(sum(recv_splits))
        gid_recv = torch.repeat_interleave(torch.arange(E_loc, device=h.device, dtype=torch.int32).repeat(ep),
                                           recv.reshape(-1).to(torch.int64), output_size=n_recv)
        lay = _layout(gid_recv, recv.sum(0), n_recv, 128)
        xe = _ScatterFn.apply(x_recv, lay, 1)
        ye = self._experts(xe, lay)
        y_recv = _GatherFn.apply(ye, None, lay, n_recv, 1)
        y_send = all_to_all(y_recv, recv_splits, send_splits, self.ep_group)
        return _GatherFn.apply(y_send, probs, send_lay, T, k), aux

    def _experts(self, xe: torch.Tensor, lay: dict) -> torch.Tensor:
        a = _GroupedLinearNativeFn.apply(xe, self.w1, lay)
        a = F_.swiglu(a)
        return _GroupedLinearNativeFn.apply(a, self.w2, lay)

    def _torch_forward(self, h: torch.Tensor):
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
