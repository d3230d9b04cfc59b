"""Context parallelism: attention over a sequence split into 2*CP load-balanced chunks.

CP rank ``r`` holds chunks ``r`` and ``2*CP-1-r`` (so every rank does the same amount of causal work).  K and
V are all-gathered over the CP group (reduce-scattered in backward) and each rank attends its queries to all
keys with a causal mask in *global* positions.  In the reference CP lives entirely in Megatron/TE
(context_parallel_size is only carried and folded into the ZeRO group, parallel_strategy.py:131-147).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import functional as F_


def _positions(seq_local: int, cp: int, r: int) -> torch.Tensor:
    c = seq_local // 2
    a = torch.arange(r * c, (r + 1) * c)
    b = torch.arange((2 * cp - 1 - r) * c, (2 * cp - r) * c)
    return torch.cat([a, b])


def cp_attention(qkv: torch.Tensor, hpg: int, group, cp_rank: int, cp: int) -> torch.Tensor:
    s, b, G, _, d = qkv.shape
    kv = qkv[:, :, :, hpg:].contiguous()  # [s, b, G, 2, d]
    kv_all = F_.gather_from_sp(kv.view(s, -1), group).view(cp * s, b, G, 2, d)
    qpos = _positions(s, cp, cp_rank).to(qkv.device)
    kpos = torch.cat([_positions(s, cp, r) for r in range(cp)]).to(qkv.device)
    mask = qpos[:, None] >= kpos[None, :]
    q = qkv[:, :, :, :hpg].reshape(s, b, G * hpg, d).permute(1, 2, 0, 3)
    k = kv_all[:, :, :, 0].permute(1, 2, 0, 3)
    v = kv_all[:, :, :, 1].permute(1, 2, 0, 3)
    if hpg > 1:
        k = k.repeat_interleave(hpg, 1)
        v = v.repeat_interleave(hpg, 1)
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    return o.permute(2, 0, 1, 3).reshape(s, b, G * hpg * d)
