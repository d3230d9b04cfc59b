"""Checkpoints in Megatron's legacy per-rank layout, loadable under any strategy.

Layout (what the reference writes through Megatron ``save_checkpoint`` with ``use_dist_ckpt=False``,
elastic_megatron/megatron_manager/training_state.py:325-366, and what tools/ckpt/compare_ckpt.py:9-14 reads)::

    <dir>/latest_checkpointed_iteration.txt
    <dir>/iter_0000010/mp_rank_TT[_PPP][_EEE]/model_optim_rng.pt    # 'model', 'args', 'iteration', ...
    <dir>/iter_0000010/mp_rank_TT[_PPP][_EEE]/distrib_optim.pt      # fp32 master / exp_avg / exp_avg_sq

``model`` holds the TP-local parameters under their local (per-stage) names; experts are written
unstacked under ``mlp.experts.local_experts.<e>.linear_fc{1,2}.weight`` with the local expert index.
``distrib_optim.pt`` holds, per parameter name, the ``[3, *shape]`` optimizer state of the whole TP-local
parameter, gathered over the data-parallel shard group (one writer per (TP, PP, EP) coordinate).

Loading under a different strategy (a resume after a re-layout) reassembles the global, layout-free tensors
from the saved strategy's files through the same index maps the planner uses, and scatters them into the
current strategy's arenas - so ``save under A, load under B`` equals a live ``reshard(A -> B)`` bit for bit.
"""
from __future__ import annotations

import os
import random
from typing import Dict, Optional

import numpy as np
import torch
import torch.distributed as dist

from ..config import get_args
from ..parallel.process_groups import ProcessGroupPool
from ..parallel.strategy import ParallelStrategy
from ..planner.layout import rank_layout, virtual_params
from ..planner.plan import _StrategyView


def checkpoint_name(root: str, iteration: int, tp: int, pp: Optional[int], ep: Optional[int]) -> str:
    d = f"mp_rank_{tp:02d}"
    if pp is not None:
        d += f"_{pp:03d}"
    if ep is not None:
        d += f"_{ep:03d}"
    return os.path.join(root, f"iter_{iteration:07d}", d)


def _dir_for(s: ParallelStrategy, rank: int, root: str, iteration: int) -> str:
    c = s.coords(rank)
    pp = c["pp"] if s.pipeline_model_parallel_size > 1 else None
    ep = c["ep"] if s.expert_model_parallel_size > 1 else None
    return checkpoint_name(root, iteration, c["tp"], pp, ep)


def _local_names(layout):
    """(state-dict name, arena offset, shape, vp) for every local tensor, experts unstacked."""
    out = []
    for lp in layout.params:
        base = layout.offset_by_name[lp.name]
        if lp.is_expert:
            shp = lp.shape[1:]
            n = int(np.prod(shp))
            for vp, off in lp.members:
                name = (f"decoder.layers.{lp.layer_local}.mlp.experts.local_experts.{off // n}."
                        + lp.key.split("mlp.experts.")[1])
                out.append((name, base + off, tuple(shp), vp))
        else:
            out.append((lp.name, base, tuple(lp.shape), lp.members[0][0]))
    return out


def _gather_opt_full(ts) -> Dict[str, torch.Tensor]:
    """[3, *shape] fp32 optimizer state of every local tensor, summed over its ZeRO shard group."""
    O = ts.opt_flat.detach().cpu()
    owned = ts.layout.owned()
    names = _local_names(ts.layout)
    res = {}
    for name, off, shp, vp in names:
        n = int(np.prod(shp))
        t = torch.zeros((3, n), dtype=torch.float32)
        for s, e, o in owned:
            lo, hi = max(s, off), min(e, off + n)
            if lo < hi:
                t[:, lo - off:hi - off] = O[:, o + (lo - s):o + (hi - s)]
        res[name] = t
    dense = [nm for nm, _, _, vp in names if not vp.is_expert]
    expert = [nm for nm, _, _, vp in names if vp.is_expert]
    for keys, gname in ((dense, "zero"), (expert, "expert_zero")):
        ranks = ts.ps.group_ranks.get(gname)
        if not keys or not dist.is_initialized() or ranks is None or len(ranks) == 1:
            continue
        flat = torch.cat([res[k].reshape(-1) for k in keys])
        if dist.get_backend() == "nccl":
            flat = flat.to(ts.device)
        dist.all_reduce(flat, group=ProcessGroupPool.get(ranks))
        flat = flat.cpu()
        o = 0
        for k in keys:
            n = res[k].numel()
            res[k] = flat[o:o + n].view_as(res[k])
            o += n
    return {nm: res[nm].view(3, *shp) for nm, _, shp, _ in names}


def save_checkpoint(ts, root: str, iteration: Optional[int] = None, consumed_samples: Optional[int] = None) -> str:
    """Collective over the strategy's ranks; one writer per (TP, PP, EP) coordinate."""
    args = get_args()
    if iteration is None:
        iteration = args.iteration
    if consumed_samples is None:
        consumed_samples = args.consumed_train_samples
    s, rank = ts.strategy, ts.rank
    opt_full = _gather_opt_full(ts)
    c = s.coords(rank)
    writer = c["dp"] == 0 and c["cp"] == 0 and ts.layout.instance == 0
    d = _dir_for(s, rank, root, iteration)
    if writer:
        os.makedirs(d, exist_ok=True)
        P = ts.param_flat.detach().cpu()
        model = {name: P[off:off + int(np.prod(shp))].view(shp).clone()
                 for name, off, shp, vp in _local_names(ts.layout)}
        state = {
            "args": {"model": dict(args.model.__dict__), "train": dict(args.train.__dict__),
                     "strategy": s.to_dict()},
            "checkpoint_version": 3.0,
            "iteration": iteration,
            "model": model,
            "optimizer": ts.optimizer.state_dict(),
            "opt_param_scheduler": ts.opt_param_scheduler.state_dict(),
            "rng_state": [{"random_rng_state": random.getstate(), "np_rng_state": np.random.get_state(),
                           "torch_rng_state": torch.get_rng_state(),
                           "cuda_rng_state": torch.cuda.get_rng_state() if torch.cuda.is_available() else None}],
            "consumed_train_samples": consumed_samples,
        }
        torch.save(state, os.path.join(d, "model_optim_rng.pt"))
        torch.save(opt_full, os.path.join(d, "distrib_optim.pt"))
    if dist.is_initialized() and s.world_size > 1:
        dist.barrier(group=ProcessGroupPool.get(s.ranks, "gloo"))
    if rank == 0:
        with open(os.path.join(root, "latest_checkpointed_iteration.txt"), "w") as f:
            f.write(str(iteration))
    return d


def read_latest(root: str) -> int:
    with open(os.path.join(root, "latest_checkpointed_iteration.txt")) as f:
        return int(f.read().strip())


def read_global_state(root: str, iteration: Optional[int] = None):
    """Reassemble layout-free global tensors from a checkpoint saved under any strategy.

    Returns ``(params, opt, meta)`` with ``params[vp.index]`` fp32 global tensors, ``opt[vp.index]`` the
    ``[3, *shape]`` master / exp_avg / exp_avg_sq, and the metadata of the first rank file.
    """
    args = get_args()
    cfg, tc = args.model, args.train
    if iteration is None:
        iteration = read_latest(root)
    it_dir = os.path.join(root, f"iter_{iteration:07d}")
    first = next(os.path.join(it_dir, sub, "model_optim_rng.pt") for sub in sorted(os.listdir(it_dir))
                 if os.path.exists(os.path.join(it_dir, sub, "model_optim_rng.pt")))
    meta = torch.load(first, weights_only=False)
    saved = ParallelStrategy(**meta["args"]["strategy"])
    vps = virtual_params(cfg)
    g_param = {vp.index: torch.zeros(vp.shape, dtype=torch.float32) for vp in vps}
    g_opt = {vp.index: torch.zeros((3,) + tuple(vp.shape), dtype=torch.float32) for vp in vps}
    view = _StrategyView(cfg, saved, tc.overlap_grad_reduce, tc.ddp_bucket_size)
    seen = set()
    for r in range(saved.world_size):
        d = _dir_for(saved, r, root, iteration)
        if d in seen or not os.path.exists(d):
            continue
        seen.add(d)
        st = torch.load(os.path.join(d, "model_optim_rng.pt"), weights_only=False)
        opt = torch.load(os.path.join(d, "distrib_optim.pt"), weights_only=False)
        # emulate rank r's param arena and a full-size optimizer arena with the same offsets
        rl = rank_layout(cfg, saved, r, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        P = torch.zeros(rl.param_numel)
        O = torch.zeros(3, rl.param_numel)
        for name, off, shp, vp in _local_names(rl):
            n = int(np.prod(shp))
            P[off:off + n] = st["model"][name].reshape(-1).float()
            O[:, off:off + n] = opt[name].reshape(3, -1)
        for vp in vps:
            if r not in view.holders(vp):
                continue
            g2 = g_param[vp.index].view(1, -1) if len(vp.shape) == 1 else g_param[vp.index]
            o2 = g_opt[vp.index].view(3, 1, -1) if len(vp.shape) == 1 else g_opt[vp.index]
            for pc in view.param_pieces(vp, r):
                k = pc.gc1 - pc.gc0
                for gr in range(pc.gr0, pc.gr1):
                    o = pc.off(gr, pc.gc0)
                    g2[gr, pc.gc0:pc.gc1] = P[o:o + k]
                    o2[:, gr, pc.gc0:pc.gc1] = O[:, o:o + k]
    meta["saved_strategy"] = saved
    return g_param, g_opt, meta


def load_checkpoint(ts, root: str, iteration: Optional[int] = None) -> Dict:
    """Load params + optimizer state (+ scheduler) saved under any strategy into ``ts``'s layout."""
    from ..planner.materialize import scatter_to_rank

    args = get_args()
    cfg, tc = args.model, args.train
    g_param, g_opt, meta = read_global_state(root, iteration)
    Pc = torch.zeros(ts.param_flat.shape, dtype=torch.float32)
    Oc = torch.zeros(ts.opt_flat.shape, dtype=torch.float32)
    scatter_to_rank(cfg, ts.strategy, ts.rank, g_param, Pc, Oc, g_opt, tc.overlap_grad_reduce, tc.ddp_bucket_size)
    ts.param_flat.copy_(Pc.to(ts.param_dtype))
    ts.opt_flat.copy_(Oc)
    ts.optimizer.load_state_dict(meta["optimizer"])
    ts.opt_param_scheduler.load_state_dict(meta["opt_param_scheduler"])
    args.iteration = meta["iteration"]
    args.consumed_train_samples = meta.get("consumed_train_samples", 0)
    return {"iteration": meta["iteration"], "saved_strategy": meta["saved_strategy"],
            "consumed_train_samples": args.consumed_train_samples}


def convert_checkpoint(src_root: str, dst_root: str, dst_strategy, iteration: Optional[int] = None) -> None:
    """Offline re-layout of a checkpoint to another strategy (one process, no process groups)."""
    from ..planner.materialize import scatter_to_rank

    args = get_args()
    cfg, tc = args.model, args.train
    g_param, g_opt, meta = read_global_state(src_root, iteration)
    dst = ParallelStrategy.from_any(dst_strategy)
    it = meta["iteration"]
    for r in range(dst.world_size):
        c = dst.coords(r)
        rl = rank_layout(cfg, dst, r, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        if not (c["dp"] == 0 and c["cp"] == 0 and rl.instance == 0):
            continue
        P = torch.zeros(rl.param_numel)
        Ofull = torch.zeros(3, rl.param_numel)
        # parameters and the whole TP-local optimizer state (written as if one rank owned every shard)
        O = torch.zeros(3, rl.opt_numel)
        scatter_to_rank(cfg, dst, r, g_param, P, O, g_opt, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        from ..planner.plan import _StrategyView

        view = _StrategyView(cfg, dst, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        for vp in virtual_params(cfg):
            if r not in view.holders(vp):
                continue
            o2 = g_opt[vp.index].view(3, 1, -1) if len(vp.shape) == 1 else g_opt[vp.index]
            for pc in view.param_pieces(vp, r):
                k = pc.gc1 - pc.gc0
                for gr in range(pc.gr0, pc.gr1):
                    o = pc.off(gr, pc.gc0)
                    Ofull[:, o:o + k] = o2[:, gr, pc.gc0:pc.gc1]
        d = _dir_for(dst, r, dst_root, it)
        os.makedirs(d, exist_ok=True)
        names = _local_names(rl)
        model = {n: P[off:off + int(np.prod(shp))].view(shp).to(cfg.torch_dtype).clone() for n, off, shp, _ in names}
        optim = {n: Ofull[:, off:off + int(np.prod(shp))].reshape(3, *shp).clone() for n, off, shp, _ in names}
        state = dict(meta)
        state.pop("saved_strategy", None)
        state["args"] = dict(meta["args"])
        state["args"]["strategy"] = dst.to_dict()
        state["model"] = model
        torch.save(state, os.path.join(d, "model_optim_rng.pt"))
        torch.save(optim, os.path.join(d, "distrib_optim.pt"))
    with open(os.path.join(dst_root, "latest_checkpointed_iteration.txt"), "w") as f:
        f.write(str(it))
