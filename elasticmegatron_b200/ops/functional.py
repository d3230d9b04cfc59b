"""Autograd functions of the training core.

Each function dispatches CUDA tensors to the native sm_100a kernels (``ops/native.py``) and CPU tensors to
``ops/reference.py``.  Linear layers accumulate their weight gradient directly into the parameter's fp32
``main_grad`` (the wgrad GEMM runs with ``C += A*B`` into the fp32 gradient buffer), so no bf16 ``.grad``
tensor is ever materialised for them; after accumulating they call the parameter's ``_grad_ready`` hook,
which the DDP layer uses to start bucket reduce-scatters.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import reference as ref
from . import tp_fused
from .native import use_native, ext


# ----------------------------------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, b: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
         out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    """``op(a) @ op(b)`` with op = transpose when ``trans_*``; ``accumulate`` adds into ``out`` (fp32 ok)."""
    if use_native(a):
        return ext().gemm(a, b, trans_a, trans_b, out, accumulate)
    A = a.t() if trans_a else a
    B = b.t() if trans_b else b
    r = torch.matmul(A.float() if out is not None and out.dtype == torch.float32 else A,
                     B.float() if out is not None and out.dtype == torch.float32 else B)
    if out is None:
        return r
    if accumulate:
        out.add_(r.to(out.dtype))
    else:
        out.copy_(r)
    return out


def _accumulate_wgrad(w: torch.nn.Parameter, dy2: torch.Tensor, x2: torch.Tensor):
    """dW[N,K] (+)= dy^T[N,M] @ x[M,K]."""
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        gemm(dy2, x2, trans_a=True, trans_b=False, out=mg.view(w.shape), accumulate=True)
        hook = getattr(w, "_grad_ready", None)
        if hook is not None:
            hook()
        return None
    return gemm(dy2, x2, trans_a=True).to(w.dtype)


# ----------------------------------------------------------------------------------------- collectives
def _all_gather_dim0(x: torch.Tensor, group) -> torch.Tensor:
    n = dist.get_world_size(group)
    if n == 1:
        return x
    out = torch.empty((n * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _reduce_scatter_dim0(x: torch.Tensor, group) -> torch.Tensor:
    n = dist.get_world_size(group)
    if n == 1:
        return x
    out = torch.empty((x.shape[0] // n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


def _all_reduce(x: torch.Tensor, group) -> torch.Tensor:
    if dist.get_world_size(group) > 1:
        dist.all_reduce(x, group=group)
    return x


class _GatherFromSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather_dim0(x, group)

    @staticmethod
    def backward(ctx, dy):
        return _reduce_scatter_dim0(dy, ctx.group), None


class _ScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n, r = dist.get_world_size(group), dist.get_rank(group)
        c = x.shape[0] // n
        return x[r * c:(r + 1) * c].contiguous()

    @staticmethod
    def backward(ctx, dy):
        return _all_gather_dim0(dy, ctx.group), None


class _ReduceScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter_dim0(x, group)

    @staticmethod
    def backward(ctx, dy):
        return _all_gather_dim0(dy, ctx.group), None


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, dy):
        return _all_reduce(dy.contiguous(), ctx.group), None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        return _all_reduce(x.contiguous(), group)

    @staticmethod
    def backward(ctx, dy):
        return dy, None


def gather_from_sp(x, group):
    return _GatherFromSP.apply(x, group) if group is not None and dist.get_world_size(group) > 1 else x


def scatter_to_sp(x, group):
    return _ScatterToSP.apply(x, group) if group is not None and dist.get_world_size(group) > 1 else x


def reduce_scatter_to_sp(x, group):
    return _ReduceScatterToSP.apply(x, group) if group is not None and dist.get_world_size(group) > 1 else x


def copy_to_tp(x, group):
    return _CopyToTP.apply(x, group) if group is not None and dist.get_world_size(group) > 1 else x


def reduce_from_tp(x, group):
    return _ReduceFromTP.apply(x, group) if group is not None and dist.get_world_size(group) > 1 else x


# ------------------------------------------------------------------------------------------ linear
class LinearFn(torch.autograd.Function):
    """y = comm_out(comm_in(x) @ W^T) with the TP/SP collective of the layer folded in.

    mode: ``None`` (no TP), ``"col"`` (column-parallel, no SP: identity fwd / all-reduce bwd), ``"row"``
    (row-parallel, no SP: all-reduce fwd), ``"col_sp"`` (all-gather seq fwd / reduce-scatter bwd),
    ``"row_sp"`` (reduce-scatter seq fwd / all-gather bwd).
    """

    @staticmethod
    def forward(ctx, x, w, mode, group):
        ctx.mode, ctx.group = mode, group
        assert x.dim() == 2, "activations are [tokens, features]"
        x2 = x
        if mode == "col_sp" and tp_fused.ag_eligible(x2, w, True, group):
            y, _ = tp_fused.all_gather_gemm(x2, w, True, group)
        elif mode == "col_sp":
            xf = _all_gather_dim0(x2, group)
            y = gemm(xf, w, trans_b=True)
        elif mode == "row_sp" and tp_fused.eligible(x2, w, False, True, group):
            y = tp_fused.gemm_reduce_scatter(x2, w, False, True, group)
        else:
            y = gemm(x2, w, trans_b=True)
            if mode == "row_sp":
                y = _reduce_scatter_dim0(y, group)
            elif mode == "row":
                y = _all_reduce(y, group)
        ctx.save_for_backward(x2, w)
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        mode, group = ctx.mode, ctx.group
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        if mode == "row_sp" and tp_fused.ag_eligible(dy2, w, False, group):
            # fused all-gather of dy with the dgrad GEMM; the gathered dy feeds the wgrad right after
            dx, dyf = tp_fused.all_gather_gemm(dy2, w, False, group)
            dw = _accumulate_wgrad(w, dyf, x2)
            return dx, dw, None, None
        if mode == "row_sp":
            dy2 = _all_gather_dim0(dy2, group)
        xf = _all_gather_dim0(x2, group) if mode == "col_sp" else x2
        if mode == "col_sp" and tp_fused.eligible(dy2, w, False, False, group):
            dx = tp_fused.gemm_reduce_scatter(dy2, w, False, False, group)
        else:
            dx = gemm(dy2, w)  # [M,N] @ [N,K]
            if mode == "col_sp":
                dx = _reduce_scatter_dim0(dx, group)
            elif mode == "col":
                dx = _all_reduce(dx, group)
        dw = _accumulate_wgrad(w, dy2, xf)
        return dx, dw, None, None


def linear(x, w, mode=None, group=None):
    if group is None or dist.get_world_size(group) == 1:
        mode = None
    return LinearFn.apply(x, w, mode, group)


# ------------------------------------------------------------------------------------------ RMSNorm
class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2 = x.reshape(-1, x.shape[-1])
        if use_native(x2):
            y, rstd = ext().rmsnorm_fwd(x2.contiguous(), w, eps)
        else:
            y, rstd = ref.rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        mg = getattr(w, "main_grad", None)
        if use_native(x2):
            # the weight gradient is reduced in fp32 straight into main_grad when the weight has one
            dx, dw = ext().rmsnorm_bwd(dy2, x2, w, rstd, mg.view(-1) if mg is not None else None)
        else:
            dx, dw = ref.rmsnorm_bwd(dy2, x2, w, rstd)
            if mg is not None:
                mg.view(-1).add_(dw)
        if mg is not None:
            hook = getattr(w, "_grad_ready", None)
            if hook is not None:
                hook()
            return dx.view(dy.shape), None, None
        return dx.view(dy.shape), dw.to(w.dtype), None


def rmsnorm(x, w, eps):
    return RMSNormFn.apply(x, w, eps)


class AddRMSNormFn(torch.autograd.Function):
    """``h = x + o`` (the residual stream) and ``y = RMSNorm(h) * w`` in one kernel; the backward adds the
    residual stream's gradient ``dh`` inside the norm's backward kernel, so neither the forward add nor the
    gradient sum at the branch point is a separate pass over the activations."""

    @staticmethod
    def forward(ctx, x, o, w, eps):
        x2, o2 = x.reshape(-1, x.shape[-1]), o.reshape(-1, o.shape[-1])
        if use_native(x2):
            h, y, rstd = ext().add_rmsnorm_fwd(x2.contiguous(), o2.contiguous(), w, eps)
        else:
            h = x2 + o2
            y, rstd = ref.rmsnorm_fwd(h, w, eps)
        ctx.save_for_backward(h, w, rstd)
        return h.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dh2 = dh.reshape(-1, dh.shape[-1]).contiguous() if dh is not None else None
        mg = getattr(w, "main_grad", None)
        if use_native(h):
            dx, dw = ext().rmsnorm_bwd(dy2, h, w, rstd, mg.view(-1) if mg is not None else None, dh2)
        else:
            dx, dw = ref.rmsnorm_bwd(dy2, h, w, rstd)
            if dh2 is not None:
                dx = dx + dh2
            if mg is not None:
                mg.view(-1).add_(dw)
        dx = dx.view(dy.shape)
        if mg is not None:
            hook = getattr(w, "_grad_ready", None)
            if hook is not None:
                hook()
            return dx, dx, None, None
        return dx, dx, dw.to(w.dtype), None


def add_rmsnorm(x, o, w, eps):
    """(x + o, RMSNorm(x + o) * w)."""
    return AddRMSNormFn.apply(x, o, w, eps)


class LayerNormFn(torch.autograd.Function):
    """LayerNorm on the native kernels (bf16 on CUDA): fp32 statistics, weight / bias gradients reduced in
    fp32 straight into ``main_grad`` when the parameters have one (as the RMSNorm path does)."""

    @staticmethod
    def forward(ctx, x, w, b, eps):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        y, mean, rstd = ext().layernorm_fwd(x2, w, b, eps)
        ctx.save_for_backward(x2, w, b, mean, rstd)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, b, mean, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        mw, mb = getattr(w, "main_grad", None), getattr(b, "main_grad", None)
        dx, dw, db = ext().layernorm_bwd(dy2, x2, w, mean, rstd, mw.view(-1) if mw is not None else None,
                                         mb.view(-1) if mb is not None else None)
        out_w, out_b = None, None
        for p, m, g in ((w, mw, dw), (b, mb, db)):
            if m is not None:
                hook = getattr(p, "_grad_ready", None)
                if hook is not None:
                    hook()
        if mw is None:
            out_w = dw.to(w.dtype)
        if mb is None:
            out_b = db.to(b.dtype)
        return dx.view(dy.shape), out_w, out_b, None


def layernorm(x, w, b, eps):
    """Megatron's LayerNorm (weight and bias) over the last dimension: the native kernels for bf16 CUDA
    tensors (hidden size a multiple of 8), PyTorch's ``layer_norm`` on the host."""
    if (use_native(x) and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0
            and hasattr(ext(), "layernorm_fwd")):
        return LayerNormFn.apply(x, w, b, eps)
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


# ------------------------------------------------------------------------------------------ SwiGLU
class SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h):
        ctx.save_for_backward(h)
        if use_native(h):
            return ext().swiglu_fwd(h.contiguous())
        return ref.swiglu_fwd(h)

    @staticmethod
    def backward(ctx, dy):
        (h,) = ctx.saved_tensors
        if use_native(h):
            return ext().swiglu_bwd(dy.contiguous(), h)
        return ref.swiglu_bwd(dy, h)


def swiglu(h):
    return SwiGLUFn.apply(h)


# ------------------------------------------------------------------------------------------ RoPE
class RoPEFn(torch.autograd.Function):
    """In: fused qkv activations [s, b, G, (hpg+2), d]; applies RoPE to the q and k slots."""

    @staticmethod
    def forward(ctx, qkv, cos, sin, nrot):
        ctx.save_for_backward(cos, sin)
        ctx.nrot = nrot
        if use_native(qkv):
            return ext().rope_fwd(qkv.contiguous(), cos, sin, nrot, False)
        out = qkv.clone()
        s, b = qkv.shape[0], qkv.shape[1]
        x = qkv[:, :, :, :nrot].reshape(s, b, -1, qkv.shape[-1])
        out[:, :, :, :nrot] = ref.rope_apply(x, cos, sin).view_as(qkv[:, :, :, :nrot])
        return out

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        nrot = ctx.nrot
        if use_native(dy):
            return ext().rope_fwd(dy.contiguous(), cos, sin, nrot, True), None, None, None
        out = dy.clone()
        s, b = dy.shape[0], dy.shape[1]
        x = dy[:, :, :, :nrot].reshape(s, b, -1, dy.shape[-1])
        out[:, :, :, :nrot] = ref.rope_apply(x, cos, sin, inverse=True).view_as(dy[:, :, :, :nrot])
        return out, None, None, None


def rope_qkv(qkv, cos, sin, nrot):
    return RoPEFn.apply(qkv, cos, sin, nrot)


# ------------------------------------------------------------------------------------------ attention
class AttentionFn(torch.autograd.Function):
    """Causal GQA attention on the fused layout [s, b, G, hpg+2, d] -> [s, b, G*hpg*d]."""

    @staticmethod
    def forward(ctx, qkv, hpg):
        s, b, G, _, d = qkv.shape
        ctx.hpg = hpg
        if use_native(qkv):
            o, lse = ext().attn_fwd(qkv.contiguous(), hpg, True)
            ctx.save_for_backward(qkv, o, lse)
            return o
        q = qkv[:, :, :, :hpg].reshape(s, b, G * hpg, d).permute(1, 2, 0, 3)
        k = qkv[:, :, :, hpg].permute(1, 2, 0, 3)
        v = qkv[:, :, :, hpg + 1].permute(1, 2, 0, 3)
        o, lse = ref.attention_fwd(q, k, v, causal=True)
        o = o.permute(2, 0, 1, 3).reshape(s, b, G * hpg * d)
        ctx.save_for_backward(qkv, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        hpg = ctx.hpg
        if use_native(qkv):
            return ext().attn_bwd(do.contiguous(), qkv, o, lse, hpg, True), None
        with torch.enable_grad():
            x = qkv.detach().requires_grad_(True)
            s, b, G, _, d = x.shape
            q = x[:, :, :, :hpg].reshape(s, b, G * hpg, d).permute(1, 2, 0, 3)
            k = x[:, :, :, hpg].permute(1, 2, 0, 3)
            v = x[:, :, :, hpg + 1].permute(1, 2, 0, 3)
            if hpg > 1:
                k = k.repeat_interleave(hpg, 1)
                v = v.repeat_interleave(hpg, 1)
            y = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
            y = y.permute(2, 0, 1, 3).reshape(s, b, -1)
            (dx,) = torch.autograd.grad(y, x, do.float())
        return dx.to(qkv.dtype), None


def _has_native_attention() -> bool:
    """The native flash attention kernels (``csrc/attn``) are the CUDA path for bf16, head dim 128 and sequence
    lengths that are multiples of 128; ``EMB_NATIVE_ATTENTION=0`` selects PyTorch SDPA (library) instead.

    Measured at the Llama-2 7B shape (s=4096, 32 heads, d=128, causal) the forward takes 0.163 ms and the backward
    0.799 ms, against 0.114 / ~0.70 ms for SDPA (cuDNN); a 7B training step is ~3 % slower than with SDPA.
    """
    import os

    if os.environ.get("EMB_NATIVE_ATTENTION", "1") == "0":
        return False
    try:
        return hasattr(ext(), "attn_bwd")
    except RuntimeError:
        return False


def _sdpa_attention(qkv, hpg):
    """Interim CUDA path for shapes the native attention kernel does not cover: PyTorch SDPA (library)."""
    s, b, G, _, d = qkv.shape
    q = qkv[:, :, :, :hpg].reshape(s, b, G * hpg, d).permute(1, 2, 0, 3)
    k = qkv[:, :, :, hpg].permute(1, 2, 0, 3)
    v = qkv[:, :, :, hpg + 1].permute(1, 2, 0, 3)
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=hpg > 1)
    return o.permute(2, 0, 1, 3).reshape(s, b, G * hpg * d)


def attention(qkv, hpg):
    if qkv.is_cuda and not (_has_native_attention() and ext().attn_supported(qkv)):
        return _sdpa_attention(qkv, hpg)
    return AttentionFn.apply(qkv, hpg)


# ------------------------------------------------------------------------------------------ vocab-parallel CE
class VocabParallelCE(torch.autograd.Function):
    """Cross-entropy over logits split along the vocab across TP ranks (fp32 math).

    logits: [T, V/tp] (any float dtype); labels: [T] global ids.  Returns per-token loss [T] fp32.
    """

    @staticmethod
    def forward(ctx, logits, labels, vocab_start, group):
        ctx.group = group
        if use_native(logits):
            # local max -> all-reduce max -> local sum-exp & target logit -> all-reduce sum
            lmax = ext().ce_local_max(logits)
            if group is not None and dist.get_world_size(group) > 1:
                dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=group)
            stats = ext().ce_local_stats(logits, labels, lmax, vocab_start)  # [2, T]: sumexp, target
            if group is not None and dist.get_world_size(group) > 1:
                dist.all_reduce(stats, group=group)
            loss = torch.log(stats[0]) - stats[1]  # stats[1] = target logit - global max
            ctx.save_for_backward(logits, labels, lmax, stats[0])
            ctx.vocab_start = vocab_start
            return loss
        lf = logits.float()
        lmax = lf.max(-1).values
        if group is not None and dist.get_world_size(group) > 1:
            dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(lf - lmax[:, None])
        sumexp = ex.sum(-1)
        V = lf.shape[-1]
        local = labels - vocab_start
        inr = (local >= 0) & (local < V)
        tgt = torch.zeros_like(lmax)
        idx = local.clamp(0, V - 1)
        tgt[inr] = lf.gather(1, idx[:, None]).squeeze(1)[inr] - lmax[inr]
        st = torch.stack([sumexp, tgt])
        if group is not None and dist.get_world_size(group) > 1:
            dist.all_reduce(st, group=group)
        loss = torch.log(st[0]) - st[1]
        ctx.save_for_backward(logits, labels, lmax, st[0])
        ctx.vocab_start = vocab_start
        return loss

    @staticmethod
    def backward(ctx, dloss):
        logits, labels, lmax, sumexp = ctx.saved_tensors
        if use_native(logits):
            return ext().ce_bwd(logits, labels, lmax, sumexp, dloss.contiguous(), ctx.vocab_start), None, None, None
        lf = logits.float()
        p = torch.exp(lf - lmax[:, None]) / sumexp[:, None]
        V = lf.shape[-1]
        local = labels - ctx.vocab_start
        inr = (local >= 0) & (local < V)
        rows = torch.nonzero(inr).squeeze(1)
        p[rows, local[rows]] -= 1.0
        return (p * dloss[:, None]).to(logits.dtype), None, None, None


def vocab_parallel_cross_entropy(logits, labels, vocab_start, group):
    return VocabParallelCE.apply(logits, labels, vocab_start, group)


# ------------------------------------------------------------------------------------------ embedding
class VocabParallelEmbedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w, vocab_start, group):
        V = w.shape[0]
        ctx.vocab_start, ctx.group = vocab_start, group
        if use_native(w):
            out = ext().embedding_fwd(ids, w, vocab_start)
        else:
            local = ids - vocab_start
            mask = (local < 0) | (local >= V)
            out = w[local.clamp(0, V - 1)]
            out[mask] = 0
        ctx.save_for_backward(ids, w)
        return out

    @staticmethod
    def backward(ctx, dy):
        ids, w = ctx.saved_tensors
        mg = getattr(w, "main_grad", None)
        target = mg.view(w.shape) if mg is not None else torch.zeros(w.shape, dtype=torch.float32,
                                                                       device=w.device)
        if use_native(w):
            ext().embedding_bwd(ids, dy.contiguous(), target, ctx.vocab_start)
        else:
            V = w.shape[0]
            local = (ids - ctx.vocab_start).reshape(-1)
            d2 = dy.reshape(-1, dy.shape[-1]).float()
            keep = (local >= 0) & (local < V)
            target.index_add_(0, local[keep], d2[keep])
        if mg is not None:
            hook = getattr(w, "_grad_ready", None)
            if hook is not None:
                hook()
            return None, None, None, None
        return None, target.to(w.dtype), None, None


def embedding(ids, w, vocab_start):
    return VocabParallelEmbedding.apply(ids, w, vocab_start, None)
