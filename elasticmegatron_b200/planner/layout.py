"""Where every element of parameter, gradient and optimizer state lives, as a pure function.

The reference recovers Megatron's ZeRO-1 shard layout by running a real ``_ParamAndGradBuffer`` constructor
over fake tensors with mocked ``torch.zeros`` / ``get_world_size`` (elastic_megatron/resharding/
resharding_dp.py:155-315).  This training core owns its buffers, so the layout is defined here once and both
the runtime (``parallel/ddp.py``) and the planner import it.  Rules:

* parameters are packed in *reverse* forward order (gradients become ready in that order);
* each parameter starts on a multiple of ``ALIGN`` elements (512-byte aligned fp32 / 256-byte bf16, so every
  kernel can use 16-byte vectors and TMA-legal addresses);
* a bucket closes once it holds ``>= bucket_size`` elements; its end is padded to a multiple of
  ``shard_group_size * ALIGN`` so all shards are equal and aligned.  ``bucket_size=None`` -> one bucket.
  The default size ``max(40M, 1M * dp)`` when gradient reduction overlaps backward matches the reference's
  rule (resharding_dp.py:332-336);
* rank ``z`` of the shard group owns ``[b.start + z*shard_b, b.start + (z+1)*shard_b)`` of every bucket ``b``;
  its optimizer buffer is the concatenation of those slices, bucket by bucket.

Dense parameters shard over the DP*CP group split into optimizer instances; expert parameters over the
expert-DP group split the same way.  A rank's flat param/grad arena is ``[dense buffer | expert buffer]`` and
its optimizer arena ``[dense shards | expert shards]``.
"""
from __future__ import annotations

import bisect
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from ..config import ModelConfig
from ..models.spec import LocalParam, VParam, build_virtual_params, local_params

ALIGN = 128


def _align(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def default_bucket_size(shard_group_size: int, overlap_grad_reduce: bool, ddp_bucket_size: Optional[int]):
    if not overlap_grad_reduce:
        return None
    if ddp_bucket_size is not None:
        return ddp_bucket_size
    return max(40_000_000, 1_000_000 * shard_group_size)


@dataclass
class BufferLayout:
    params: List[LocalParam]
    param_ranges: List[Tuple[int, int]]  # per param (start, end) in this buffer
    buckets: List[Tuple[int, int]]
    bucket_params: List[List[int]]  # param indices (in ``params``) per bucket
    shard_group_size: int
    numel: int

    def shard_size(self, b: int) -> int:
        s, e = self.buckets[b]
        return (e - s) // self.shard_group_size

    def owned_ranges(self, z: int) -> List[Tuple[int, int, int]]:
        """(buffer_start, buffer_end, optimizer_offset) owned by shard index ``z``."""
        out, opt = [], 0
        for b, (s, _) in enumerate(self.buckets):
            n = self.shard_size(b)
            out.append((s + z * n, s + (z + 1) * n, opt))
            opt += n
        return out

    @property
    def opt_numel(self) -> int:
        return sum(self.shard_size(b) for b in range(len(self.buckets)))


def build_buffer_layout(params: List[LocalParam], shard_group_size: int,
                        bucket_size: Optional[int]) -> BufferLayout:
    ranges: List[Tuple[int, int]] = [(0, 0)] * len(params)
    buckets, bparams = [], []
    cur, bstart, members = 0, 0, []
    gran = shard_group_size * ALIGN

    def close():
        nonlocal cur, bstart, members
        end = _align(cur, gran)
        if end == bstart:
            end = bstart + gran
        buckets.append((bstart, end))
        bparams.append(members)
        cur = end
        bstart = end
        members = []

    for i in reversed(range(len(params))):
        start = _align(cur, ALIGN)
        ranges[i] = (start, start + params[i].numel)
        cur = start + params[i].numel
        members.append(i)
        if bucket_size is not None and cur - bstart >= bucket_size:
            close()
    if members or not buckets:
        close()
    return BufferLayout(params=params, param_ranges=ranges, buckets=buckets, bucket_params=bparams,
                        shard_group_size=shard_group_size, numel=buckets[-1][1] if buckets else 0)


@dataclass
class RankLayout:
    """Everything about one rank's state under one strategy."""

    rank: int
    params: List[LocalParam]  # forward order, dense and expert mixed
    dense: BufferLayout
    expert: Optional[BufferLayout]
    dense_shard_index: int
    expert_shard_index: Optional[int]
    instance: int
    # virtual-param index -> (arena offset of its local shard, local shard shape)
    vp_loc: Dict[int, Tuple[int, Tuple[int, ...]]] = field(default_factory=dict)
    offset_by_name: Dict[str, int] = field(default_factory=dict)
    _owned: Optional[List[Tuple[int, int, int]]] = field(default=None, repr=False, compare=False)
    _owned_starts: Optional[List[int]] = field(default=None, repr=False, compare=False)

    def __post_init__(self):
        for i, lp in enumerate(self.dense.params):
            self.offset_by_name[lp.name] = self.dense.param_ranges[i][0]
        if self.expert is not None:
            for i, lp in enumerate(self.expert.params):
                self.offset_by_name[lp.name] = self.dense.numel + self.expert.param_ranges[i][0]
        for lp in self.params:
            base = self.offset_by_name[lp.name]
            shp = lp.shape[1:] if lp.is_expert else lp.shape
            for vp, off in lp.members:
                self.vp_loc[vp.index] = (base + off, tuple(shp))

    @property
    def param_numel(self) -> int:
        return self.dense.numel + (self.expert.numel if self.expert else 0)

    @property
    def opt_numel(self) -> int:
        return self.dense.opt_numel + (self.expert.opt_numel if self.expert else 0)

    def param_offset(self, lp: LocalParam) -> int:
        """Start of ``lp`` in the rank's flat param arena."""
        return self.offset_by_name[lp.name]

    def owned(self) -> List[Tuple[int, int, int]]:
        """(arena_start, arena_end, opt_offset) of every owned optimizer slice (dense then expert), in arena
        order; computed once per layout (layouts are cached, and the planner asks per parameter)."""
        if self._owned is None:
            out = list(self.dense.owned_ranges(self.dense_shard_index))
            if self.expert is not None:
                base_p, base_o = self.dense.numel, self.dense.opt_numel
                out += [(s + base_p, e + base_p, o + base_o)
                        for s, e, o in self.expert.owned_ranges(self.expert_shard_index)]
            self._owned = out
            self._owned_starts = [s for s, _, _ in out]
        return list(self._owned)

    def owned_overlapping(self, a: int, b: int) -> List[Tuple[int, int, int]]:
        """The owned slices that intersect the arena range ``[a, b)`` (binary search; slices are disjoint and
        sorted)."""
        self.owned()
        i = max(0, bisect.bisect_right(self._owned_starts, a) - 1)
        out = []
        while i < len(self._owned) and self._owned[i][0] < b:
            s, e, o = self._owned[i]
            if e > a:
                out.append((s, e, o))
            i += 1
        return out


def _cfg_key(cfg: ModelConfig):
    return tuple(sorted(cfg.__dict__.items()))


_VP_CACHE: Dict[tuple, List[VParam]] = {}


def virtual_params(cfg: ModelConfig) -> List[VParam]:
    k = _cfg_key(cfg)
    if k not in _VP_CACHE:
        _VP_CACHE[k] = build_virtual_params(cfg)
    return _VP_CACHE[k]


_RL_CACHE: Dict[tuple, RankLayout] = {}


def rank_layout(cfg: ModelConfig, strategy, rank: int, overlap_grad_reduce: bool = False,
                ddp_bucket_size: Optional[int] = None) -> RankLayout:
    key = (_cfg_key(cfg), strategy.key(), rank, overlap_grad_reduce, ddp_bucket_size)
    rl = _RL_CACHE.get(key)
    if rl is not None:
        return rl
    vps = virtual_params(cfg)
    lps = local_params(cfg, vps, strategy, rank)
    dense_p = [p for p in lps if not p.is_expert]
    exp_p = [p for p in lps if p.is_expert]
    z = strategy.zero_coords(rank)
    dense = build_buffer_layout(dense_p, z["dense_shard_size"],
                                default_bucket_size(z["dense_shard_size"], overlap_grad_reduce, ddp_bucket_size))
    expert = None
    if exp_p:
        expert = build_buffer_layout(exp_p, z["expert_shard_size"],
                                     default_bucket_size(z["expert_shard_size"], overlap_grad_reduce,
                                                         ddp_bucket_size))
    rl = RankLayout(rank=rank, params=lps, dense=dense, expert=expert, dense_shard_index=z["dense_shard"],
                    expert_shard_index=z["expert_shard"] if exp_p else None, instance=z["dense_instance"])
    _RL_CACHE[key] = rl
    return rl
