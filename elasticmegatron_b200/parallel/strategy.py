"""``ParallelStrategy``: the unit of configuration that a job switches between.

Same fields, defaults and derivation rules as the reference's dataclass
(elastic_megatron/megatron_manager/parallel_strategy.py:10-49):

* ``DP = world_size / (TP * PP * CP)``; ``sequence_parallel`` defaults to ``TP > 1`` and is rejected with TP 1;
* ``expert_tensor_parallel_size`` defaults to TP; ``expert-DP = world_size / (ETP * EP * PP)``;
* transformer layers are split uniformly over PP stages, experts uniformly over EP ranks;
* active ranks are always the prefix ``0 .. world_size-1`` (``is_running = rank < world_size``).

Differences by design:

* every coordinate accessor takes an optional ``rank`` so the planner can reason about *any* rank of a
  strategy without process groups (the reference reads them from Megatron's live ``parallel_state``);
* ``sequence_parallel`` is part of the strategy identity (the reference excludes it from ``__str__`` /
  ``__hash__``, :223-232, so two strategies differing only in SP collide);
* Group-ZeRO (``num_distributed_optimizer_instances > 1``) does not require CP > 1: that constraint is a
  Megatron 0.11 limitation (:99-106) which this training core does not have.
"""
from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Dict, List, Optional

from ..config import get_args
from .rank_generator import ElasticRankGenerator


def _current_rank() -> int:
    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            return dist.get_rank()
    except Exception:  # pragma: no cover
        pass
    return 0


@dataclass
class ParallelStrategy:
    world_size: int
    tensor_model_parallel_size: int
    pipeline_model_parallel_size: int
    context_parallel_size: int = 1
    num_distributed_optimizer_instances: int = 1
    expert_model_parallel_size: int = 1
    expert_tensor_parallel_size: Optional[int] = None
    sequence_parallel: Optional[bool] = None
    order: str = "tp-cp-ep-dp-pp"
    ranks: Optional[List[int]] = None

    def __post_init__(self):
        self._rank = _current_rank()
        self.is_running = self._rank < self.world_size
        assert self.world_size > 0
        tp, pp, cp = self.tensor_model_parallel_size, self.pipeline_model_parallel_size, self.context_parallel_size
        assert self.world_size % tp == 0, f"world_size {self.world_size} not divisible by TP {tp}"
        assert self.world_size % pp == 0, f"world_size {self.world_size} not divisible by PP {pp}"
        self.model_parallel_size = tp * pp
        self.total_model_size = self.model_parallel_size * cp
        assert self.world_size % self.total_model_size == 0
        self.data_parallel_size = self.world_size // self.total_model_size
        if tp == 1 and self.sequence_parallel:
            raise ValueError("sequence_parallel=True needs tensor_model_parallel_size > 1 (SP splits the sequence over the TP group)")
        if self.sequence_parallel is None:
            self.sequence_parallel = tp > 1
        if self.ranks is None:
            self.ranks = list(range(self.world_size))
        # Group-ZeRO
        inst = self.num_distributed_optimizer_instances
        assert inst >= 1
        assert (self.data_parallel_size * cp) % inst == 0, "DP*CP must divide by the optimizer instance count"
        # MoE mesh
        if self.expert_tensor_parallel_size is None:
            self.expert_tensor_parallel_size = tp
        etpp = self.expert_tensor_parallel_size * self.expert_model_parallel_size * pp
        if self.world_size % etpp != 0:
            raise RuntimeError(f"world_size ({self.world_size}) is not divisible by ETP*EP*PP ({etpp})")
        self.expert_data_parallel_size = self.world_size // etpp
        # layers / experts
        args = get_args()
        self.num_layers = args.num_layers
        assert self.num_layers >= 1 and self.num_layers % pp == 0, \
            f"num_layers {self.num_layers} must divide by PP {pp}"
        self.transformer_layer_num_per_stage = self.num_layers // pp
        self.num_experts = args.num_experts or None
        if self.num_experts:
            assert self.num_experts % self.expert_model_parallel_size == 0
            self.expert_num_per_ep_rank = self.num_experts // self.expert_model_parallel_size
            assert self.expert_tensor_parallel_size == 1, "Only ETP==1 is supported for MoE resharding"
            if tp > 1:
                assert self.sequence_parallel, "MoE with TP > 1 requires sequence parallelism"
        else:
            self.expert_num_per_ep_rank = None
        self.rank_generator = ElasticRankGenerator(self)

    # ------------------------------------------------------------------ identity
    def key(self) -> tuple:
        return (self.world_size, self.tensor_model_parallel_size, self.pipeline_model_parallel_size,
                self.context_parallel_size, self.num_distributed_optimizer_instances,
                self.expert_model_parallel_size, self.expert_tensor_parallel_size, bool(self.sequence_parallel),
                self.order)

    def layout_key(self) -> tuple:
        """Everything that determines where state lives (SP does not)."""
        return self.key()[:7] + (self.order,)

    def __str__(self):
        return (f"ws{self.world_size}-tp{self.tensor_model_parallel_size}-pp{self.pipeline_model_parallel_size}"
                f"-cp{self.context_parallel_size}-dp{self.data_parallel_size}-ep{self.expert_model_parallel_size}"
                f"-etp{self.expert_tensor_parallel_size}-inst{self.num_distributed_optimizer_instances}"
                f"{'-sp' if self.sequence_parallel else ('-nosp' if self.tensor_model_parallel_size > 1 else '')}")

    def __repr__(self):
        return f"ParallelStrategy({self})"

    def __hash__(self):
        return hash(self.key())

    def __eq__(self, other):
        return isinstance(other, ParallelStrategy) and self.key() == other.key()

    def to_dict(self) -> Dict:
        return {f.name: getattr(self, f.name) for f in fields(self) if f.name != "ranks"}

    @classmethod
    def from_any(cls, s) -> "ParallelStrategy":
        if isinstance(s, ParallelStrategy):
            return s
        if isinstance(s, str):
            return cls.parse(s)
        return cls(**s)

    _SPEC_KEYS = {"ws": "world_size", "tp": "tensor_model_parallel_size", "pp": "pipeline_model_parallel_size",
                  "cp": "context_parallel_size", "ep": "expert_model_parallel_size",
                  "etp": "expert_tensor_parallel_size", "inst": "num_distributed_optimizer_instances"}

    @classmethod
    def parse(cls, spec: str) -> "ParallelStrategy":
        """Inverse of ``str()``: ``"ws8-tp2-pp1"``, ``"ws4-tp2-sp"``, ``"ws8-ep4"`` ... (missing sizes default
        to 1; ``dp`` is derived and ignored if given; ``sp`` / ``nosp`` force sequence parallelism)."""
        kw: Dict = {"tensor_model_parallel_size": 1, "pipeline_model_parallel_size": 1}
        for tok in spec.strip().split("-"):
            if tok in ("sp", "nosp"):
                kw["sequence_parallel"] = tok == "sp"
                continue
            key = tok.rstrip("0123456789")
            if key == "dp":
                continue
            if key not in cls._SPEC_KEYS or key == tok:
                raise ValueError(f"bad strategy token {tok!r} in {spec!r}")
            kw[cls._SPEC_KEYS[key]] = int(tok[len(key):])
        if "world_size" not in kw:
            raise ValueError(f"strategy {spec!r} needs a ws<N> token")
        return cls(**kw)

    # ------------------------------------------------------------------ coordinates
    def coords(self, rank: Optional[int] = None) -> Dict[str, int]:
        """Dense-mesh coordinates (tp, cp, dp, pp) and expert-mesh coordinates (etp, ep, edp) of ``rank``."""
        rank = self._rank if rank is None else rank
        assert 0 <= rank < self.world_size, f"rank {rank} outside strategy {self}"
        d = self.rank_generator.dense.coords_of(rank)
        e = self.rank_generator.expert.coords_of(rank)
        return {"tp": d["tp"], "cp": d["cp"], "dp": d["dp"], "pp": d["pp"],
                "etp": e["tp"], "ep": e["ep"], "edp": e["dp"]}

    def rank_of(self, tp=0, cp=0, dp=0, pp=0) -> int:
        return self.rank_generator.dense.rank_of(tp=tp, cp=cp, dp=dp, pp=pp)

    def expert_rank_of(self, etp=0, ep=0, edp=0, pp=0) -> int:
        return self.rank_generator.expert.rank_of(tp=etp, ep=ep, dp=edp, pp=pp)

    def get_ranks(self, group_type: str, is_expert: bool = False, rank: Optional[int] = None) -> Optional[List[int]]:
        rank = self._rank if rank is None else rank
        for ranks in self.rank_generator.get_ranks(group_type, is_expert):
            if rank in ranks:
                return ranks
        return None

    def all_groups(self, group_type: str, is_expert: bool = False) -> List[List[int]]:
        return self.rank_generator.get_ranks(group_type, is_expert)

    # per-process convenience (reference: register_mpu_state, :149-188)
    @property
    def tensor_model_parallel_rank(self):
        return self.coords()["tp"]

    @property
    def pipeline_model_parallel_rank(self):
        return self.coords()["pp"]

    @property
    def data_parallel_rank(self):
        return self.coords()["dp"]

    @property
    def context_parallel_rank(self):
        return self.coords()["cp"]

    @property
    def expert_model_parallel_rank(self):
        return self.coords()["ep"] if self.num_experts else None

    @property
    def expert_tensor_parallel_rank(self):
        return self.coords()["etp"] if self.num_experts else None

    @property
    def expert_data_parallel_rank(self):
        return self.coords()["edp"] if self.num_experts else None

    def get_tensor_model_parallel_size(self, is_expert: bool) -> int:
        return self.expert_tensor_parallel_size if is_expert else self.tensor_model_parallel_size

    def get_tensor_model_parallel_rank(self, is_expert: bool, rank: Optional[int] = None) -> int:
        c = self.coords(rank)
        return c["etp"] if is_expert else c["tp"]

    @property
    def transformer_layer_id_offset(self):
        return self.transformer_layer_num_per_stage * self.pipeline_model_parallel_rank

    @property
    def expert_id_offset(self):
        return self.expert_num_per_ep_rank * self.coords()["ep"]

    def get_data_parallel_world_size(self, with_context_parallel: bool = False,
                                     partial_data_parallel: bool = False) -> int:
        if with_context_parallel:
            n = self.data_parallel_size * self.context_parallel_size
            if partial_data_parallel:
                return n // self.num_distributed_optimizer_instances
            return n
        assert not partial_data_parallel, "Partial DP for the optimizer needs to include CP"
        return self.data_parallel_size

    @property
    def zero_shard_size(self) -> int:
        """Number of ranks one dense optimizer shard group spans (DP*CP / instances)."""
        return self.get_data_parallel_world_size(True, True)

    @property
    def expert_zero_shard_size(self) -> int:
        return self.expert_data_parallel_size // self.num_distributed_optimizer_instances

    def zero_coords(self, rank: Optional[int] = None) -> Dict[str, int]:
        """Position of ``rank`` in its dense and expert optimizer-shard groups and its instance index.

        The dense shard group of a rank is its DP*CP group split into ``instances`` contiguous pieces;
        the expert shard group is its expert-DP group split the same way.
        """
        rank = self._rank if rank is None else rank
        inst = self.num_distributed_optimizer_instances
        dpcp = self.get_ranks("cp-dp", rank=rank)
        i = dpcp.index(rank)
        n = len(dpcp) // inst
        out = {"dense_shard": i % n, "dense_instance": i // n, "dense_shard_size": n}
        edp = self.get_ranks("dp", is_expert=True, rank=rank)
        j = edp.index(rank)
        m = len(edp) // inst
        out.update({"expert_shard": j % m, "expert_instance": j // m, "expert_shard_size": m})
        return out

    def check_consistency(self, other: "ParallelStrategy") -> None:
        for k in ("world_size", "tensor_model_parallel_size", "pipeline_model_parallel_size",
                  "context_parallel_size", "sequence_parallel", "num_distributed_optimizer_instances"):
            assert getattr(self, k) == getattr(other, k), f"{k}: {getattr(self, k)} != {getattr(other, k)}"

    @staticmethod
    def is_redundant_backup(src: "ParallelStrategy", dst: "ParallelStrategy") -> Optional[bool]:
        """Classify a switch (elastic_megatron/megatron_manager/parallel_strategy.py:234-263).

        Returns ``None`` for an ordinary re-layout, ``True`` for a Group-ZeRO scale-up (more optimizer
        replicas), ``False`` for a Group-ZeRO scale-down.
        """
        sg, dg = src.num_distributed_optimizer_instances, dst.num_distributed_optimizer_instances
        if sg == dg:
            if sg != 1:
                raise ValueError(f"both layouts keep {sg} optimizer instances: a switch that keeps the Group-ZeRO instance "
                                 "count above 1 is not implemented")
            return None
        assert src.model_parallel_size == dst.model_parallel_size
        assert src.context_parallel_size == dst.context_parallel_size
        assert src.world_size != dst.world_size
        assert src.world_size * dg == dst.world_size * sg
        return sg < dg


def union_ranks(a: ParallelStrategy, b: ParallelStrategy) -> List[int]:
    return sorted(set(a.ranks) | set(b.ranks))
