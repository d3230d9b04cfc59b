"""Plain-PyTorch implementations of every hot op.

These are (1) the CPU path used by gloo-rank tests and (2) the fp32 oracles every CUDA kernel is tested
against.  They are never used for CUDA tensors: the dispatch in ``ops/functional.py`` raises if the native
extension is missing on a GPU.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (xf * rstd * w.float()).to(x.dtype)
    return y, rstd.squeeze(-1)


def rmsnorm_bwd(dy, x, w, rstd) -> Tuple[torch.Tensor, torch.Tensor]:
    xf, dyf, wf = x.float(), dy.float(), w.float()
    r = rstd.unsqueeze(-1)
    xhat = xf * r
    dw = (dyf * xhat).reshape(-1, x.shape[-1]).sum(0)
    g = dyf * wf
    dx = r * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    return dx.to(x.dtype), dw


def rope_cos_sin(positions: torch.Tensor, dim: int, base: float):
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64, device=positions.device) / dim))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return ang.cos().float(), ang.sin().float()


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """x: [s, b, n, d] rotate-half convention on pairs (i, i + d/2); cos/sin: [s, d/2]."""
    d2 = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :d2], xf[..., d2:]
    c = cos[:, None, None, :]
    s = sin[:, None, None, :]
    if inverse:
        s = -s
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)


def swiglu_fwd(h: torch.Tensor) -> torch.Tensor:
    """h: [..., 2f] = [gate | up] -> silu(gate) * up."""
    g, u = h.float().chunk(2, -1)
    return (F.silu(g) * u).to(h.dtype)


def swiglu_bwd(dy: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    g, u = h.float().chunk(2, -1)
    dyf = dy.float()
    sg = torch.sigmoid(g)
    silu = g * sg
    dg = dyf * u * (sg * (1 + g * (1 - sg)))
    du = dyf * silu
    return torch.cat([dg, du], -1).to(h.dtype)


def attention_fwd(q, k, v, causal: bool = True, scale: Optional[float] = None):
    """q: [b, hq, s, d], k/v: [b, hkv, t, d] (GQA) -> (o [b,hq,s,d], lse [b,hq,s] fp32)."""
    hq, hkv = q.shape[1], k.shape[1]
    if hq != hkv:
        k = k.repeat_interleave(hq // hkv, 1)
        v = v.repeat_interleave(hq // hkv, 1)
    scale = scale or 1.0 / math.sqrt(q.shape[-1])
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        S, T = q.shape[2], k.shape[2]
        mask = torch.ones(S, T, dtype=torch.bool, device=q.device).tril(T - S)
        s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse.unsqueeze(-1))
    o = torch.matmul(p, v.float())
    return o.to(q.dtype), lse


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return F.cross_entropy(logits.float(), labels, reduction="none")


def adam_step(master, exp_avg, exp_avg_sq, grad, lr, beta1, beta2, eps, wd, step, clip_coef=1.0):
    """Decoupled AdamW with bias correction on fp32 tensors, in place (torch.optim.AdamW semantics)."""
    g = grad.float() * clip_coef
    exp_avg.mul_(beta1).add_(g, alpha=1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (exp_avg_sq / bc2).sqrt_().add_(eps)
    if wd != 0.0:
        master.mul_(1 - lr * wd)
    master.addcdiv_(exp_avg, denom, value=-lr / bc1)
