"""Context parallelism: attention over a sequence split into 2*CP load-balanced chunks.

CP rank ``r`` holds chunks ``r`` and ``2*CP-1-r`` (so every rank does the same amount of causal work).  K and
V are all-gathered over the CP group (reduce-scattered in backward); each query chunk attends to the global
prefix of keys that ends with its own chunk.  In the reference CP lives entirely in Megatron/TE
(context_parallel_size is only carried and folded into the ZeRO group, parallel_strategy.py:131-147).
"""
from __future__ import annotations

import torch

from ..ops import functional as F_


def _global_chunk_starts(s: int, cp: int):
    """Row offset, inside the rank-ordered all-gather of K/V, of every global chunk 0 .. 2*CP-1."""
    c = s // 2
    out = []
    for g in range(2 * cp):
        r, half = (g, 0) if g < cp else (2 * cp - 1 - g, 1)
        out.append(r * s + half * c)
    return out


def cp_attention(qkv: torch.Tensor, hpg: int, group, cp_rank: int, cp: int) -> torch.Tensor:
    """Causal attention of this rank's two query chunks against the gathered keys / values.

    K / V are all-gathered in rank order and re-ordered into global sequence order; query chunk ``ci`` then
    attends to the global prefix ``[0, (ci + 1) * c)`` with a causal mask aligned to the lower right (its
    own chunk is the last block of that prefix), so each chunk is one fused attention call with no explicit
    mask tensor and no K/V head replication (grouped-query attention is native to the call)."""
    from torch.nn.attention.bias import causal_lower_right

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
