"""Checkpoints in Megatron's legacy per-rank layout, loadable under any strategy.

Layout (what the reference writes through Megatron ``save_checkpoint`` with ``use_dist_ckpt=False``,
elastic_megatron/megatron_manager/training_state.py:325-366, and what tools/ckpt/compare_ckpt.py:9-14 reads)::

    <dir>/latest_checkpointed_iteration.txt
    <dir>/iter_0000010/mp_rank_TT[_PPP][_EEE]/model_optim_rng.pt    # 'model', 'args', 'iteration', ...
    <dir>/iter_0000010/mp_rank_TT[_PPP][_EEE]/distrib_optim.pt      # fp32 master / exp_avg / exp_avg_sq

``model`` holds the TP-local parameters under their local (per-stage) names; experts are written
unstacked under ``mlp.experts.local_experts.<e>.linear_fc{1,2}.weight`` with the local expert index.  One rank
writes each (TP, PP, EP) directory: the lowest rank with that coordinate in optimizer instance 0 (Megatron
writes from expert-data-parallel rank 0), so every expert shard is saved once.

``distrib_optim.pt`` uses the coalesced format of Megatron's ``DistributedOptimizer.save_parameter_state``
(``get_parameter_state_dp_zero``): ``{"buckets_coalesced": True, buffer: {(param dtype, grad dtype):
{"param", "exp_avg", "exp_avg_sq", "numel_unpadded"}}}`` where each tensor is the fp32 state flat over the
grad buffer, bucket by bucket, with each bucket's end padding removed.  Buffer 0 is the dense buffer (written
in the ep == 0 directory of its (TP, PP)), buffer 1 the expert buffer.  The shards are gathered onto the
writer one bucket at a time over the ZeRO group, so no other rank ever holds the full state.  The positions
inside a buffer follow this framework's layout rules (``planner/layout.py``), recorded under ``emb_layout``.

Loading under a different strategy (a resume after a re-layout) reassembles the global, layout-free tensors
from the saved strategy's files through the same index maps the planner uses, and scatters them into the
current strategy's arenas - so ``save under A, load under B`` equals a live ``reshard(A -> B)`` bit for bit.
"""
from __future__ import annotations

import os
import random
from typing import Dict, List, Optional, Tuple

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


def _file_key(s: ParallelStrategy, rank: int) -> Tuple[int, Optional[int], Optional[int]]:
    """(tp, pp, ep) coordinate that names ``rank``'s checkpoint directory (pp / ep None when not split)."""
    c = s.coords(rank)
    return (c["tp"], c["pp"] if s.pipeline_model_parallel_size > 1 else None,
            c["ep"] if s.expert_model_parallel_size > 1 else None)


def _dense_key(key):
    """The directory that holds the dense optimizer state of ``key``'s (tp, pp): the ep == 0 one."""
    return (key[0], key[1], 0 if key[2] is not None else None)


def _writers(s: ParallelStrategy) -> Dict[tuple, int]:
    """One writer rank per (tp, pp, ep) directory: the lowest rank with that coordinate in optimizer instance 0.

    Experts are carved out of the dense data-parallel dimension, so ranks that share a dense coordinate can hold
    different experts; keying the writer on the expert coordinate too (Megatron writes from expert-data-parallel
    rank 0) makes every expert shard land in its own ``mp_rank_TT[_PPP]_EEE`` directory exactly once.
    """
    out: Dict[tuple, int] = {}
    for r in range(s.world_size):
        z = s.zero_coords(r)
        if z["dense_instance"] != 0 or z["expert_instance"] != 0:
            continue
        out.setdefault(_file_key(s, r), r)
    keys = {_file_key(s, r) for r in range(s.world_size)}
    missing = keys - set(out)
    assert not missing, f"no instance-0 writer for checkpoint directories {sorted(missing)} under {s}"
    return out


def _bucket_unpadded(bl, b: int) -> int:
    """Elements of bucket ``b`` up to the end of its last parameter (the padding after it is not saved)."""
    s, _ = bl.buckets[b]
    ends = [bl.param_ranges[i][1] for i in bl.bucket_params[b]]
    return (max(ends) - s) if ends else 0


def _buffer_state_from_arena(bl, base: int, O: torch.Tensor) -> Dict:
    """Megatron's per-buffer dict (``param`` / ``exp_avg`` / ``exp_avg_sq`` flat over the buffer with each
    bucket's end padding removed, plus ``numel_unpadded``) from a full ``[3, param_numel]`` state laid out like
    the param arena (``base`` = start of this buffer in the arena)."""
    parts = []
    for b, (s, _) in enumerate(bl.buckets):
        u = _bucket_unpadded(bl, b)
        parts.append(O[:, base + s:base + s + u])
    flat = torch.cat(parts, dim=1) if parts else torch.zeros(3, 0)
    return {"param": flat[0].clone(), "exp_avg": flat[1].clone(), "exp_avg_sq": flat[2].clone(),
            "numel_unpadded": int(flat.shape[1])}


def _buffer_state_into_arena(bl, base: int, st: Dict, O: torch.Tensor) -> None:
    """Inverse of ``_buffer_state_from_arena``."""
    cum = 0
    flat = torch.stack([st["param"], st["exp_avg"], st["exp_avg_sq"]]).float()
    if int(st["numel_unpadded"]) != flat.shape[1]:
        raise ValueError(f"distrib_optim buffer: numel_unpadded {st['numel_unpadded']} != {flat.shape[1]}")
    for b, (s, _) in enumerate(bl.buckets):
        u = _bucket_unpadded(bl, b)
        O[:, base + s:base + s + u] = flat[:, cum:cum + u]
        cum += u
    if cum != flat.shape[1]:
        raise ValueError(f"distrib_optim buffer holds {flat.shape[1]} elements, the layout expects {cum}; the file "
                         f"was written under a different model or bucket configuration")


def _gather_buffer(ts, which: str, group: List[int], target: int) -> Optional[Dict]:
    """Gather one buffer's optimizer shards onto ``target`` bucket by bucket, the way Megatron's
    ``get_parameter_state_dp_zero`` does: only the target ever holds more than one bucket of other ranks'
    state, and it keeps the result on the host.  Collective over ``group`` (this rank's ZeRO shard group)."""
    lay = ts.layout
    bl = lay.dense if which == "dense" else lay.expert
    base_o = 0 if which == "dense" else lay.dense.opt_numel
    me = ts.rank
    G = len(group)
    pg = ProcessGroupPool.get(group) if G > 1 else None
    out = [] if me == target else None
    o = base_o
    for b in range(len(bl.buckets)):
        n = bl.shard_size(b)
        mine = ts.opt_flat[:, o:o + n].contiguous()
        o += n
        if G == 1:
            parts = [mine]
        else:
            parts = [torch.empty_like(mine) for _ in range(G)] if me == target else None
            dist.gather(mine, parts, dst=target, group=pg)
        if me == target:
            full = torch.stack(parts, dim=1).reshape(3, G * n)  # shard z owns [z*n, (z+1)*n) of the bucket
            out.append(full[:, :_bucket_unpadded(bl, b)].cpu())
    if me != target:
        return None
    flat = torch.cat(out, dim=1) if out else torch.zeros(3, 0)
    return {"param": flat[0].clone(), "exp_avg": flat[1].clone(), "exp_avg_sq": flat[2].clone(),
            "numel_unpadded": int(flat.shape[1])}


def _optim_file(dense: Optional[Dict], expert: Optional[Dict], param_dtype) -> Dict:
    """``distrib_optim.pt`` contents: Megatron's coalesced dp-zero format (buffer index -> {(param dtype, grad
    dtype): buffer state}); buffer 0 is the dense buffer (present in the ep == 0 directory only), buffer 1 the
    expert buffer.  ``emb_layout`` records the in-buffer layout rules the flat tensors follow."""
    from ..planner.layout import ALIGN

    d: Dict = {"buckets_coalesced": True,
               "emb_layout": {"align": ALIGN, "order": "reverse forward", "buffers": ["dense", "expert"]}}
    key = (param_dtype, torch.float32)
    if dense is not None:
        d[0] = {key: dense}
    if expert is not None:
        d[1] = {key: expert}
    return d


def _buffer_entry(optim: Dict, idx: int) -> Optional[Dict]:
    e = optim.get(idx)
    if e is None:
        return None
    return next(iter(e.values()))


def save_checkpoint(ts, root: str, iteration: Optional[int] = None, consumed_samples: Optional[int] = None) -> str:
    """Collective over the strategy's ranks; one writer per (TP, PP, EP) directory."""
    args = get_args()
    if iteration is None:
        iteration = args.iteration
    if consumed_samples is None:
        consumed_samples = args.consumed_train_samples
    s, rank = ts.strategy, ts.rank
    writers = _writers(s)
    key = _file_key(s, rank)
    z = s.zero_coords(rank)
    # dense optimizer state: one gather per instance-0 dense shard group, onto the writer of its ep == 0 directory
    dense_state = expert_state = None
    if z["dense_instance"] == 0:
        group = ts.ps.group_ranks["zero"]
        target = writers[_dense_key(key)]
        assert target in group, (target, group)
        dense_state = _gather_buffer(ts, "dense", group, target)
    if ts.layout.expert is not None and z["expert_instance"] == 0:
        group = ts.ps.group_ranks["expert_zero"]
        # every writer in this expert shard group needs the group's expert state (more than one when the
        # expert tensor-parallel size differs from the dense one); same order on every member
        for target in sorted({writers[_file_key(s, r)] for r in group} & set(group)):
            st = _gather_buffer(ts, "expert", group, target)
            if st is not None:
                expert_state = st
    d = _dir_for(s, rank, root, iteration)
    if writers[key] == rank:
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
        torch.save(_optim_file(dense_state if _dense_key(key) == key else None, expert_state, ts.param_dtype),
                   os.path.join(d, "distrib_optim.pt"))
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
    ``[3, *shape]`` master / exp_avg / exp_avg_sq, and the metadata of the first rank file.  Every (TP, PP, EP)
    directory of the saved strategy must exist: a missing one raises instead of leaving its parameters zero.
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
    writers = _writers(saved)
    optims: Dict[tuple, Dict] = {}

    def load_optim(key):
        if key not in optims:
            d = _dir_for(saved, writers[key], root, iteration)
            f = os.path.join(d, "distrib_optim.pt")
            if not os.path.exists(f):
                raise FileNotFoundError(f"checkpoint {it_dir} saved under {saved} lacks {f}")
            optims[key] = torch.load(f, weights_only=False)
        return optims[key]

    for key, r in sorted(writers.items(), key=lambda kv: kv[1]):
        d = _dir_for(saved, r, root, iteration)
        mf = os.path.join(d, "model_optim_rng.pt")
        if not os.path.exists(mf):
            raise FileNotFoundError(f"checkpoint {it_dir} saved under {saved} lacks {mf} (rank {r}'s directory)")
        st = torch.load(mf, weights_only=False)
        # emulate rank r's param arena and a full-size optimizer arena with the same offsets
        rl = rank_layout(cfg, saved, r, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        P = torch.zeros(rl.param_numel)
        O = torch.zeros(3, rl.param_numel)
        for name, off, shp, vp in _local_names(rl):
            n = int(np.prod(shp))
            P[off:off + n] = st["model"][name].reshape(-1).float()
        dense = _buffer_entry(load_optim(_dense_key(key)), 0)
        if dense is None:
            raise ValueError(f"{_dir_for(saved, writers[_dense_key(key)], root, iteration)}/distrib_optim.pt has no "
                             f"dense buffer state")
        _buffer_state_into_arena(rl.dense, 0, dense, O)
        if rl.expert is not None:
            ex = _buffer_entry(load_optim(key), 1)
            if ex is None:
                raise ValueError(f"{d}/distrib_optim.pt has no expert buffer state")
            _buffer_state_into_arena(rl.expert, rl.dense.numel, ex, O)
        for vp in vps:
            if _file_key(saved, r) != key or r not in view.holders(vp):
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
    view = _StrategyView(cfg, dst, tc.overlap_grad_reduce, tc.ddp_bucket_size)
    for key, r in sorted(_writers(dst).items(), key=lambda kv: kv[1]):
        rl = rank_layout(cfg, dst, r, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        P = torch.zeros(rl.param_numel)
        scatter_to_rank(cfg, dst, r, g_param, P, None, None, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        # the whole TP-local optimizer state, laid out like the param arena (as if one rank owned every shard)
        Ofull = torch.zeros(3, rl.param_numel)
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
        dense = _buffer_state_from_arena(rl.dense, 0, Ofull) if _dense_key(key) == key else None
        expert = _buffer_state_from_arena(rl.expert, rl.dense.numel, Ofull) if rl.expert is not None else None
        state = dict(meta)
        state.pop("saved_strategy", None)
        state["args"] = dict(meta["args"])
        state["args"]["strategy"] = dst.to_dict()
        state["model"] = model
        torch.save(state, os.path.join(d, "model_optim_rng.pt"))
        torch.save(_optim_file(dense, expert, cfg.torch_dtype), os.path.join(d, "distrib_optim.pt"))
    with open(os.path.join(dst_root, "latest_checkpointed_iteration.txt"), "w") as f:
        f.write(str(it))
