"""Move state between global (TP=PP=EP=1) tensors and one rank's flat arenas.

Used for: random-init of a model under any strategy from one global seed, checkpoint save/load across
strategies (gather to global on save, scatter on load), and as the oracle the transfer engines are tested
against.  It walks the same pieces as the planner, so it shares its index maps.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from ..config import ModelConfig
from .plan import _StrategyView


def _global2d(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(1, -1) if t.dim() == 1 else t.reshape(-1, t.shape[-1])


def scatter_to_rank(cfg: ModelConfig, strategy, rank: int, globals_: Dict[int, torch.Tensor],
                    param_arena: Optional[torch.Tensor] = None, opt_arena: Optional[torch.Tensor] = None,
                    opt_globals: Optional[Dict[int, torch.Tensor]] = None, overlap: bool = False,
                    bucket: Optional[int] = None) -> None:
    """Fill a rank's arenas from global tensors.

    ``globals_[vp.index]`` is the global parameter (fp32); ``opt_globals[vp.index]`` is a ``[3, *shape]``
    tensor of (master, exp_avg, exp_avg_sq) - if omitted the master is the global parameter and the moments
    are zero.
    """
    sv = _StrategyView(cfg, strategy, overlap, bucket)
    from .layout import virtual_params

    for vp in virtual_params(cfg):
        if rank not in sv.holders(vp):
            continue
        g = _global2d(globals_[vp.index])
        if param_arena is not None:
            for p in sv.param_pieces(vp, rank):
                blk = g[p.gr0:p.gr1, p.gc0:p.gc1]
                for i, gr in enumerate(range(p.gr0, p.gr1)):
                    o = p.off(gr, p.gc0)
                    param_arena[o:o + blk.shape[1]].copy_(blk[i])
        if opt_arena is not None:
            og = None
            if opt_globals is not None:
                og = opt_globals[vp.index].reshape(3, *g.shape)
            for p in sv.opt_pieces(vp, rank):
                for gr in range(p.gr0, p.gr1):
                    o = p.off(gr, p.gc0)
                    n = p.gc1 - p.gc0
                    if og is None:
                        opt_arena[0, o:o + n].copy_(g[gr, p.gc0:p.gc1])
                        opt_arena[1:, o:o + n].zero_()
                    else:
                        opt_arena[:, o:o + n].copy_(og[:, gr, p.gc0:p.gc1])


def gather_from_rank(cfg: ModelConfig, strategy, rank: int, out_param: Dict[int, torch.Tensor],
                     out_opt: Optional[Dict[int, torch.Tensor]], param_arena: Optional[torch.Tensor],
                     opt_arena: Optional[torch.Tensor], overlap: bool = False, bucket: Optional[int] = None) -> None:
    """Write the pieces this rank holds into global tensors (inverse of :func:`scatter_to_rank`)."""
    sv = _StrategyView(cfg, strategy, overlap, bucket)
    from .layout import virtual_params

    for vp in virtual_params(cfg):
        if rank not in sv.holders(vp):
            continue
        if param_arena is not None and vp.index in out_param:
            g = _global2d(out_param[vp.index])
            for p in sv.param_pieces(vp, rank):
                for gr in range(p.gr0, p.gr1):
                    o = p.off(gr, p.gc0)
                    g[gr, p.gc0:p.gc1].copy_(param_arena[o:o + p.gc1 - p.gc0])
        if opt_arena is not None and out_opt is not None and vp.index in out_opt:
            og = out_opt[vp.index]
            og2 = og.reshape(3, -1, vp.shape[-1]) if len(vp.shape) > 1 else og.reshape(3, 1, -1)
            for p in sv.opt_pieces(vp, rank):
                for gr in range(p.gr0, p.gr1):
                    o = p.off(gr, p.gc0)
                    og2[:, gr, p.gc0:p.gc1].copy_(opt_arena[:, o:o + p.gc1 - p.gc0])


def init_global_params(cfg: ModelConfig, seed: int = 0, dtype=torch.float32) -> Dict[int, torch.Tensor]:
    """N(0, std) weights and unit norm weights, generated per virtual param from one seed (layout-free)."""
    from .layout import virtual_params

    out = {}
    for vp in virtual_params(cfg):
        g = torch.Generator().manual_seed(seed * 1_000_003 + vp.index)
        if vp.init == "ones":
            out[vp.index] = torch.ones(vp.shape, dtype=dtype)
        elif vp.init == "zeros":
            out[vp.index] = torch.zeros(vp.shape, dtype=dtype)
        else:
            out[vp.index] = torch.randn(vp.shape, generator=g, dtype=torch.float32).mul_(
                cfg.init_method_std).to(dtype)
    return out
