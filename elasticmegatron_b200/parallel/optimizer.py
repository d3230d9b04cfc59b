"""Distributed AdamW over ZeRO-1 shards (with Group-ZeRO replicas).

State per rank: one fp32 ``[3, n]`` optimizer arena holding (master weight, exp_avg, exp_avg_sq) for the
rank's own shard of every bucket (``planner/layout.py``).  One step:

1. global grad L2 norm over the own shards (TP-duplicated params counted on TP rank 0 only, Group-ZeRO
   replicas on instance 0 only), all-reduced over the strategy's ranks;
2. fused AdamW on the shard with the ``1/(DP*CP)`` gradient scale and the clip coefficient folded in, writing
   the new parameter (cast to the param dtype) straight into the shard of the parameter arena;
3. the DDP layer all-gathers the parameter buckets.

This is the role Megatron's DistributedOptimizer plays for the reference (master/exp_avg/exp_avg_sq lookup at
elastic_megatron/resharding/resharding_metadata.py:208-284; ``_copy_main_params_to_model_params`` +
``start_param_sync`` at training_state.py:176-197).  Adam semantics are decoupled weight decay with bias
correction; 1-D parameters (norms) get no weight decay, as in Megatron's default ``no_weight_decay_cond``.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from ..ops import reference as ref
from ..ops.native import use_native, ext
from ..planner.layout import RankLayout


def _segments(layout: RankLayout, tp_rank: int, instance: int) -> List[Tuple[int, int, int, bool, bool]]:
    """Own-shard segments as (arena_start, opt_offset, length, weight_decay, counted_in_norm).

    Padding between parameters joins a neighbouring segment: its state is all zeros and AdamW keeps zeros
    at zero, so segments stay few and long.
    """
    spans = []
    for lp in layout.params:
        off = layout.offset_by_name[lp.name]
        vp = lp.members[0][0]
        dup = (not lp.is_expert) and vp.tp_dim is None and tp_rank != 0
        # the last stage's copy of a tied embedding holds the same values and gradient as the first stage's
        dup = dup or lp.replica
        spans.append((off, off + lp.numel, (bool(lp.weight_decay), (not dup) and instance == 0)))
    spans.sort()
    segs: List[Tuple[int, int, int, bool, bool]] = []
    for s, e, o in layout.owned():
        pieces = []
        cur, last = s, None
        for a, b, flags in spans:
            if b <= s or a >= e:
                continue
            a2, b2 = max(a, s), min(b, e)
            if a2 > cur:
                pieces.append([cur, a2, last or flags])
            pieces.append([a2, b2, flags])
            cur, last = b2, flags
        if cur < e:
            pieces.append([cur, e, last or (True, False)])
        merged = []
        for a, b, f in pieces:
            if merged and merged[-1][2] == f and merged[-1][1] == a:
                merged[-1][1] = b
            else:
                merged.append([a, b, f])
        for a, b, (wd, c) in merged:
            segs.append((a, o + (a - s), b - a, wd, c))
    return segs


class DistributedAdam:
    def __init__(self, layout: RankLayout, pstate, param_arena: torch.Tensor, grad_arena: torch.Tensor,
                 opt_arena: Optional[torch.Tensor], train_cfg):
        self.layout, self.ps, self.cfg = layout, pstate, train_cfg
        self.param_arena, self.grad_arena, self.opt_arena = param_arena, grad_arena, opt_arena
        s = pstate.strategy
        self.grad_scale = 1.0 / (s.data_parallel_size * s.context_parallel_size)
        self.segs = _segments(layout, pstate.tp_rank, layout.instance)
        self._seg_table = None
        # Two param groups (decay / no decay) for scheduler and checkpoint compatibility.
        self.param_groups = [
            {"lr": train_cfg.lr, "weight_decay": train_cfg.weight_decay, "step": 0,
             "betas": (train_cfg.adam_beta1, train_cfg.adam_beta2), "eps": train_cfg.adam_eps},
            {"lr": train_cfg.lr, "weight_decay": 0.0, "step": 0,
             "betas": (train_cfg.adam_beta1, train_cfg.adam_beta2), "eps": train_cfg.adam_eps},
        ]

    def bind(self, param_arena, grad_arena, opt_arena):
        self.param_arena, self.grad_arena, self.opt_arena = param_arena, grad_arena, opt_arena
        self._seg_table = None

    @property
    def step_count(self) -> int:
        return self.param_groups[0]["step"]

    CHUNK = 1 << 16

    def _table(self, device):
        """Segments split into chunks of at most CHUNK elements: one CTA per chunk in the native kernels."""
        if self._seg_table is None or self._seg_table.device != device:
            rows = []
            for a, o, n, wd, c in self.segs:
                for s0 in range(0, n, self.CHUNK):
                    k = min(self.CHUNK, n - s0)
                    rows.append((a + s0, o + s0, k, int(wd), int(c)))
            arr = np.array(rows, dtype=np.int64).reshape(-1, 5)
            self._seg_table = torch.from_numpy(arr).to(device)
        return self._seg_table

    def _sumsq(self) -> torch.Tensor:
        """All-reduced sum of squares of the counted own-shard gradients, as a 1-element fp32 tensor."""
        g = self.grad_arena
        if use_native(g):
            sq = ext().seg_sumsq(g, self._table(g.device))
        else:
            acc = torch.zeros((), dtype=torch.float64)
            for a, o, n, wd, c in self.segs:
                if c:
                    acc += g[a:a + n].double().pow(2).sum()
            sq = acc.float().reshape(1)
        world = self.ps.group("world")
        if world is not None and dist.get_world_size(world) > 1:
            dist.all_reduce(sq, group=world)
        return sq

    def grad_norm(self) -> float:
        return math.sqrt(float(self._sumsq().item())) * self.grad_scale

    def step(self):
        """One AdamW step.  Returns (update_successful, grad_norm); on CUDA the norm is a device tensor and the
        clip coefficient is applied inside the kernel, so the step does not synchronise with the host."""
        cfg = self.cfg
        sq = self._sumsq()
        for g in self.param_groups:
            g["step"] += 1
        step = self.param_groups[0]["step"]
        lr = self.param_groups[0]["lr"]
        b1, b2 = cfg.adam_beta1, cfg.adam_beta2
        O, G, P = self.opt_arena, self.grad_arena, self.param_arena
        max_norm = float(cfg.clip_grad or 0.0)
        if use_native(O):
            ext().adam_segments(O, G, P, self._table(O.device), lr, b1, b2, cfg.adam_eps, cfg.weight_decay, step,
                                self.grad_scale, max_norm, sq)
            return True, sq.sqrt() * self.grad_scale
        norm = math.sqrt(float(sq.item())) * self.grad_scale
        clip = 1.0
        if max_norm > 0:
            clip = min(1.0, max_norm / (norm + 1e-6))
        gscale = self.grad_scale * clip
        for a, o, n, wd, c in self.segs:
            m, ea, es = O[0, o:o + n], O[1, o:o + n], O[2, o:o + n]
            ref.adam_step(m, ea, es, G[a:a + n], lr, b1, b2, cfg.adam_eps, cfg.weight_decay if wd else 0.0,
                          step, gscale)
            P[a:a + n].copy_(m.to(P.dtype))
        return True, norm

    # ------------------------------------------------------------------ state
    def state_dict(self) -> Dict:
        return {"param_groups": [{k: v for k, v in g.items()} for g in self.param_groups]}

    def load_state_dict(self, sd: Dict) -> None:
        for g, s in zip(self.param_groups, sd["param_groups"]):
            g.update(s)
