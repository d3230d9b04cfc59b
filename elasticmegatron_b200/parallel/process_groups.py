"""Process-group pool shared by every declared strategy.

Reference behaviour (elastic_megatron/distributed/elastic_process_group.py:84-256):

* groups are de-duplicated by ``(frozenset(ranks), backend)``;
* every group of every declared strategy is created up front, collectively on all launched ranks,
  including ranks that are idle under a strategy (:216-232);
* a WORLD Gloo group backs a host barrier (:141-145, :207-210);
* NCCL groups can be destroyed and re-created to free NCCL memory (:200-205).

Here the list of groups is a pure function of the strategy list, so no ``all_gather_object`` is needed
to agree on it: every rank computes the same sorted list and creates the groups in that order.

:class:`ParallelState` is the per-strategy bundle of groups (the reference snapshots Megatron's
``parallel_state`` module globals per strategy instead, elastic_megatron/megatron_manager/mpu_state.py:7-93).
"""
from __future__ import annotations

import contextlib
import datetime
import os
from typing import Dict, FrozenSet, Iterable, List, Optional, Tuple

import torch
import torch.distributed as dist

from .strategy import ParallelStrategy

GroupKey = Tuple[FrozenSet[int], str]


def _default_backend() -> str:
    return dist.get_backend() if dist.is_initialized() else "gloo"


class _ProcessGroupPool:
    def __init__(self):
        self._groups: Dict[GroupKey, object] = {}
        self._ranks: Dict[GroupKey, List[int]] = {}
        self._gloo_world = None
        self.timeout = datetime.timedelta(seconds=float(os.environ.get("EMB200_PG_TIMEOUT_S", "600")))

    # -------------------------------------------------------------- creation
    def get(self, ranks: Iterable[int], backend: Optional[str] = None):
        """Return the cached group for ``ranks`` (must have been created collectively)."""
        ranks = sorted(ranks)
        backend = backend or _default_backend()
        key = (frozenset(ranks), backend)
        if len(ranks) == dist.get_world_size():
            if backend == _default_backend():
                return dist.group.WORLD
            if backend == "gloo":
                return self.gloo_world()
        return self._groups.get(key)

    def create(self, rank_lists: Iterable[Iterable[int]], backend: Optional[str] = None) -> None:
        """Collectively create every not-yet-existing group in ``rank_lists`` (all ranks must call)."""
        backend = backend or _default_backend()
        world = dist.get_world_size()
        todo = set()
        for rl in rank_lists:
            rl = tuple(sorted(rl))
            if len(rl) == world and (backend == _default_backend() or backend == "gloo"):
                continue
            key = (frozenset(rl), backend)
            if key not in self._groups:
                todo.add(rl)
        for rl in sorted(todo, key=lambda r: (len(r), r)):
            pg = dist.new_group(list(rl), backend=backend, timeout=self.timeout)
            key = (frozenset(rl), backend)
            self._groups[key] = pg
            self._ranks[key] = list(rl)

    def gloo_world(self):
        if self._gloo_world is None:
            if _default_backend() == "gloo":
                self._gloo_world = dist.group.WORLD
            else:
                self._gloo_world = dist.new_group(backend="gloo", timeout=self.timeout)
        return self._gloo_world

    def barrier_by_gloo(self) -> None:
        """Host barrier over every launched rank (reference: global_barrier_by_gloo, all_reduce of 1 float)."""
        t = torch.zeros(1)
        dist.all_reduce(t, group=self.gloo_world())

    def recreate_nccl_groups(self) -> None:
        """Destroy and re-create every cached NCCL group (frees NCCL buffers; all ranks must call)."""
        import sys

        tp_fused = sys.modules.get("elasticmegatron_b200.ops.tp_fused")
        if tp_fused is not None:
            tp_fused.release_buffers()  # symmetric buffers belong to the old communicators
        nvls = sys.modules.get("elasticmegatron_b200.parallel.nvls")
        if nvls is not None:
            nvls.release()  # so do the multicast staging buffers (rendezvoused on the old groups)
        keys = sorted([k for k in self._groups if k[1] == "nccl"], key=lambda k: (len(k[0]), sorted(k[0])))
        for k in keys:
            pg = self._groups.pop(k)
            if dist.get_rank() in k[0]:
                dist.destroy_process_group(pg)
        self.create([sorted(k[0]) for k in keys], backend="nccl")

    def clear(self) -> None:
        self._groups.clear()
        self._ranks.clear()
        self._gloo_world = None


ProcessGroupPool = _ProcessGroupPool()


def global_barrier_by_gloo() -> None:
    ProcessGroupPool.barrier_by_gloo()


def nccl_group_recreate() -> None:
    ProcessGroupPool.recreate_nccl_groups()


# ---------------------------------------------------------------------------------------------------------
GROUP_TOKENS = {
    # name: (token, is_expert)
    "tp": ("tp", False),
    "pp": ("pp", False),
    "dp": ("dp", False),
    "cp": ("cp", False),
    "dp_cp": ("cp-dp", False),
    "mp": ("tp-pp", False),
    "tp_cp": ("tp-cp", False),
    "ep": ("ep", True),
    "etp": ("tp", True),
    "edp": ("dp", True),
}


def strategy_rank_lists(s: ParallelStrategy) -> List[List[int]]:
    """Every rank set the strategy needs a communicator for."""
    out: List[List[int]] = [list(range(s.world_size))]
    for name, (tok, is_expert) in GROUP_TOKENS.items():
        if is_expert and not s.num_experts:
            continue
        out.extend(s.all_groups(tok, is_expert))
    out.extend(_embedding_groups(s))
    for a, b in _zero_groups(s):
        out.extend(a)
        out.extend(b)
    return [sorted(r) for r in out]


def _embedding_groups(s: ParallelStrategy) -> List[List[int]]:
    groups = []
    for pp_ranks in s.all_groups("pp"):
        groups.append(sorted({pp_ranks[0], pp_ranks[-1]}))
    return groups


def _zero_groups(s: ParallelStrategy):
    """(intra-instance shard groups, inter-instance replica groups) for the dense and expert meshes."""
    inst = s.num_distributed_optimizer_instances
    dense_intra, dense_inter, exp_intra, exp_inter = [], [], [], []
    for g in s.all_groups("cp-dp"):
        n = len(g) // inst
        dense_intra += [g[i * n:(i + 1) * n] for i in range(inst)]
        dense_inter += [g[j::n] for j in range(n)]
    if s.num_experts:
        for g in s.all_groups("dp", True):
            n = len(g) // inst
            exp_intra += [g[i * n:(i + 1) * n] for i in range(inst)]
            exp_inter += [g[j::n] for j in range(n)]
    return (dense_intra, dense_inter), (exp_intra, exp_inter)


class ParallelState:
    """Process groups and coordinates of the calling rank under one strategy."""

    def __init__(self, strategy: ParallelStrategy, backend: Optional[str] = None):
        self.strategy = strategy
        self.backend = backend or _default_backend()
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.is_running = self.rank < strategy.world_size
        self.groups: Dict[str, object] = {}
        self.group_ranks: Dict[str, List[int]] = {}
        if not self.is_running:
            return
        s = strategy
        for name, (tok, is_expert) in GROUP_TOKENS.items():
            if is_expert and not s.num_experts:
                continue
            self._set(name, s.get_ranks(tok, is_expert))
        self._set("world", list(range(s.world_size)))
        pp = self.group_ranks["pp"]
        self._set("embedding", sorted({pp[0], pp[-1]}))
        (di, dx), (ei, ex) = _zero_groups(s)
        self._set("zero", next(g for g in di if self.rank in g))
        self._set("zero_inter", next(g for g in dx if self.rank in g))
        if s.num_experts:
            self._set("expert_zero", next(g for g in ei if self.rank in g))
            self._set("expert_zero_inter", next(g for g in ex if self.rank in g))
        c = s.coords(self.rank)
        self.tp_rank, self.pp_rank, self.dp_rank, self.cp_rank = c["tp"], c["pp"], c["dp"], c["cp"]
        self.ep_rank, self.edp_rank = c["ep"], c["edp"]
        self.tp_size = s.tensor_model_parallel_size
        self.pp_size = s.pipeline_model_parallel_size
        self.dp_size = s.data_parallel_size
        self.cp_size = s.context_parallel_size
        self.ep_size = s.expert_model_parallel_size

    def _set(self, name: str, ranks: List[int]):
        self.group_ranks[name] = ranks
        self.groups[name] = ProcessGroupPool.get(ranks, self.backend) if dist.is_initialized() else None
        if dist.is_initialized() and len(ranks) > 1 and self.groups[name] is None:
            raise RuntimeError(
                f"no {self.backend} process group for ranks {ranks} ({name} of {self.strategy}); create the groups of "
                f"every strategy first, on all ranks: create_all_groups([...]) or ElasticMegatronManager(...)")

    def group(self, name: str):
        return self.groups[name]

    def size(self, name: str) -> int:
        return len(self.group_ranks[name])

    def index(self, name: str) -> int:
        return self.group_ranks[name].index(self.rank)

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    @property
    def prev_rank(self) -> int:
        return self.group_ranks["pp"][self.pp_rank - 1]

    @property
    def next_rank(self) -> int:
        return self.group_ranks["pp"][self.pp_rank + 1]


def create_all_groups(strategies: List[ParallelStrategy], backend: Optional[str] = None,
                      extra: Iterable[Iterable[int]] = ()) -> None:
    """Create, collectively on every launched rank, the groups of all strategies plus their unions."""
    lists: List[List[int]] = []
    for s in strategies:
        lists += strategy_rank_lists(s)
    for a in strategies:
        for b in strategies:
            lists.append(sorted(set(a.ranks) | set(b.ranks)))
    lists += [list(r) for r in extra]
    ProcessGroupPool.create(lists, backend=backend)
    # host-side groups (object broadcasts, MAX of timings) for every strategy world and union
    host = [list(s.ranks) for s in strategies]
    host += [sorted(set(a.ranks) | set(b.ranks)) for a in strategies for b in strategies]
    ProcessGroupPool.create(host, backend="gloo")
    ProcessGroupPool.gloo_world()


# ---------------------------------------------------------------------------------------------------------
# Optional torch.distributed default-group patch (reference: elastic_megatron/distributed/dist_patch.py:8-97).
# With the patch active, collectives called without ``group=`` act on the *active strategy's* world group
# instead of all launched ranks.  Opt-in here (the reference applies it at import time).
_ACTIVE_WORLD = None
_PATCHED = {}


def set_world_group(group) -> None:
    global _ACTIVE_WORLD
    _ACTIVE_WORLD = group


def get_world_group():
    return _ACTIVE_WORLD


@contextlib.contextmanager
def with_world_group(group):
    global _ACTIVE_WORLD
    old = _ACTIVE_WORLD
    _ACTIVE_WORLD = group
    try:
        yield
    finally:
        _ACTIVE_WORLD = old


def _has_group_param(fn) -> bool:
    import inspect

    try:
        return "group" in inspect.signature(fn).parameters
    except (TypeError, ValueError):
        return False


def patch_torch_distributed() -> None:
    import functools
    import inspect

    names = [n for n in dir(dist) if not n.startswith("_") and callable(getattr(dist, n))
             and inspect.isfunction(getattr(dist, n)) and _has_group_param(getattr(dist, n))]
    for n in names:
        if n in _PATCHED:
            continue
        fn = getattr(dist, n)
        sig = inspect.signature(fn)

        @functools.wraps(fn)
        def wrapper(*args, __fn=fn, __sig=sig, **kwargs):
            if _ACTIVE_WORLD is not None:
                bound = __sig.bind_partial(*args, **kwargs)
                if bound.arguments.get("group", None) is None:
                    bound.arguments["group"] = _ACTIVE_WORLD
                    return __fn(*bound.args, **bound.kwargs)
            return __fn(*args, **kwargs)

        _PATCHED[n] = fn
        setattr(dist, n, wrapper)


def unpatch_torch_distributed() -> None:
    for n, fn in _PATCHED.items():
        setattr(dist, n, fn)
    _PATCHED.clear()
