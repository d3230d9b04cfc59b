"""The extension's main kernels as PyTorch operators (namespace ``emb``) with fake implementations.

``torch.ops.emb.<name>`` runs the sm_100a kernel on CUDA tensors and, on meta / fake tensors, only computes
the output shapes and dtypes.  That lets code built on these kernels be shape-checked, traced or built on the
``meta`` device (the reference builds its inter-process successor model on meta,
elastic_megatron/megatron_manager/meta_device_context.py:40-240) without a GPU or a launch.  The framework's own
autograd functions call the extension directly; these registrations are for callers that want operators.

Registered: ``gemm``, ``gemm_grouped``, ``rmsnorm_fwd``, ``rmsnorm_bwd``, ``swiglu_fwd``, ``swiglu_bwd``,
``rope_fwd``, ``ce_local_max``, ``ce_local_stats``, ``embedding_fwd``, ``attn_fwd``.
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor
from torch.library import custom_op


def _ext():
    from .native import ext

    return ext()


@custom_op("emb::gemm", mutates_args=(), device_types="cuda")
def gemm(a: Tensor, b: Tensor, trans_a: bool, trans_b: bool) -> Tensor:
    return _ext().gemm(a, b, trans_a, trans_b)


@gemm.register_fake
def _(a, b, trans_a, trans_b):
    M = a.shape[1] if trans_a else a.shape[0]
    N = b.shape[0] if trans_b else b.shape[1]
    return a.new_empty((M, N))


@custom_op("emb::gemm_grouped", mutates_args=(), device_types="cuda")
def gemm_grouped(a: Tensor, w: Tensor, trans_b: bool, tile_group: Tensor) -> Tensor:
    return _ext().gemm_grouped(a, w, trans_b, tile_group)


@gemm_grouped.register_fake
def _(a, w, trans_b, tile_group):
    return a.new_empty((a.shape[0], w.shape[1] if trans_b else w.shape[2]))


@custom_op("emb::rmsnorm_fwd", mutates_args=(), device_types="cuda")
def rmsnorm_fwd(x: Tensor, w: Tensor, eps: float) -> Tuple[Tensor, Tensor]:
    y, rstd = _ext().rmsnorm_fwd(x, w, eps)
    return y, rstd


@rmsnorm_fwd.register_fake
def _(x, w, eps):
    return x.new_empty(x.shape), x.new_empty((x.shape[0],), dtype=torch.float32)


@custom_op("emb::rmsnorm_bwd", mutates_args=(), device_types="cuda")
def rmsnorm_bwd(dy: Tensor, x: Tensor, w: Tensor, rstd: Tensor) -> Tuple[Tensor, Tensor]:
    dx, dw = _ext().rmsnorm_bwd(dy, x, w, rstd)
    return dx, dw


@rmsnorm_bwd.register_fake
def _(dy, x, w, rstd):
    return x.new_empty(x.shape), x.new_empty((x.shape[1],), dtype=torch.float32)


@custom_op("emb::swiglu_fwd", mutates_args=(), device_types="cuda")
def swiglu_fwd(h: Tensor) -> Tensor:
    return _ext().swiglu_fwd(h)


@swiglu_fwd.register_fake
def _(h):
    return h.new_empty(tuple(h.shape[:-1]) + (h.shape[-1] // 2,))


@custom_op("emb::swiglu_bwd", mutates_args=(), device_types="cuda")
def swiglu_bwd(dy: Tensor, h: Tensor) -> Tensor:
    return _ext().swiglu_bwd(dy, h)


@swiglu_bwd.register_fake
def _(dy, h):
    return h.new_empty(h.shape)


@custom_op("emb::rope_fwd", mutates_args=(), device_types="cuda")
def rope_fwd(qkv: Tensor, cos: Tensor, sin: Tensor, nrot: int, inverse: bool) -> Tensor:
    return _ext().rope_fwd(qkv, cos, sin, nrot, inverse)


@rope_fwd.register_fake
def _(qkv, cos, sin, nrot, inverse):
    return qkv.new_empty(qkv.shape)


@custom_op("emb::ce_local_max", mutates_args=(), device_types="cuda")
def ce_local_max(logits: Tensor) -> Tensor:
    return _ext().ce_local_max(logits)


@ce_local_max.register_fake
def _(logits):
    return logits.new_empty((logits.shape[0],), dtype=torch.float32)


@custom_op("emb::ce_local_stats", mutates_args=(), device_types="cuda")
def ce_local_stats(logits: Tensor, labels: Tensor, lmax: Tensor, vstart: int) -> Tensor:
    return _ext().ce_local_stats(logits, labels, lmax, vstart)


@ce_local_stats.register_fake
def _(logits, labels, lmax, vstart):
    return logits.new_empty((2, logits.shape[0]), dtype=torch.float32)


@custom_op("emb::embedding_fwd", mutates_args=(), device_types="cuda")
def embedding_fwd(ids: Tensor, w: Tensor, vstart: int) -> Tensor:
    return _ext().embedding_fwd(ids, w, vstart)


@embedding_fwd.register_fake
def _(ids, w, vstart):
    return w.new_empty((ids.numel(), w.shape[1]))


@custom_op("emb::attn_fwd", mutates_args=(), device_types="cuda")
def attn_fwd(qkv: Tensor, hpg: int, causal: bool) -> Tuple[Tensor, Tensor]:
    o, lse = _ext().attn_fwd(qkv, hpg, causal)
    return o, lse


@attn_fwd.register_fake
def _(qkv, hpg, causal):
    s, b, G, _, d = qkv.shape
    return qkv.new_empty((s, b, G * hpg * d)), qkv.new_empty((b, G * hpg, s), dtype=torch.float32)
