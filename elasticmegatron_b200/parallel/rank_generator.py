"""Rank meshes for the dense and expert parts of a model.

A strategy lays ranks out on an orthogonal grid whose axes are named by ``order`` (default
``"tp-cp-ep-dp-pp"``, first axis fastest-varying), the same convention the reference inherits from
Megatron's ``RankGenerator`` (elastic_megatron/megatron_manager/rank_generator.py:9-52).  The dense mesh has
``ep == 1``; the expert mesh has ``cp == 1``, ``tp == etp`` and ``dp == expert-dp``.

``get_ranks("tp-pp")`` returns every group obtained by fixing all axes *not* named in the token and
letting the named axes vary; inside a group the ranks are enumerated with the first named axis fastest,
and groups are enumerated with the first un-named axis fastest.
"""
from __future__ import annotations

from itertools import product
from typing import Dict, List


class RankGenerator:
    AXES = ("tp", "cp", "ep", "dp", "pp")

    def __init__(self, tp: int, ep: int, dp: int, pp: int, cp: int, order: str = "tp-cp-ep-dp-pp",
                 rank_offset: int = 0):
        self.sizes: Dict[str, int] = {"tp": tp, "ep": ep, "dp": dp, "pp": pp, "cp": cp}
        self.order: List[str] = order.lower().split("-")
        for ax in self.AXES:
            if ax not in self.order:
                if self.sizes[ax] != 1:
                    raise RuntimeError(f"axis {ax} has size {self.sizes[ax]} but is missing from order {order}")
                self.order.append(ax)
        self.world_size = 1
        for ax in self.order:
            self.world_size *= self.sizes[ax]
        self.rank_offset = rank_offset
        # stride of each axis in the linear rank
        self.stride: Dict[str, int] = {}
        s = 1
        for ax in self.order:
            self.stride[ax] = s
            s *= self.sizes[ax]

    def rank_of(self, **coords: int) -> int:
        r = 0
        for ax in self.order:
            c = coords.get(ax, 0)
            assert 0 <= c < self.sizes[ax], (ax, c, self.sizes[ax])
            r += c * self.stride[ax]
        return r + self.rank_offset

    def coords_of(self, rank: int) -> Dict[str, int]:
        rank -= self.rank_offset
        out = {}
        for ax in self.order:
            out[ax] = rank // self.stride[ax] % self.sizes[ax]
        return out

    def get_ranks(self, token: str) -> List[List[int]]:
        named = token.lower().split("-")
        for ax in named:
            assert ax in self.sizes, f"unknown axis {ax}"
        # the named axes are enumerated in mesh order (first mesh axis fastest) whatever order the token spells
        # them in, as Megatron does
        masked = [ax for ax in self.order if ax in named]
        unmasked = [ax for ax in self.order if ax not in named]
        groups = []
        # outer loop over un-named axes with the first one fastest
        for outer in product(*[range(self.sizes[ax]) for ax in reversed(unmasked)]):
            fixed = dict(zip(reversed(unmasked), outer))
            ranks = []
            for inner in product(*[range(self.sizes[ax]) for ax in reversed(masked)]):
                c = dict(fixed)
                c.update(dict(zip(reversed(masked), inner)))
                ranks.append(self.rank_of(**c))
            groups.append(ranks)
        return groups


class ElasticRankGenerator:
    """Dense + expert meshes of one strategy (elastic_megatron/megatron_manager/rank_generator.py:9-52)."""

    def __init__(self, strategy) -> None:
        self.dense = RankGenerator(tp=strategy.tensor_model_parallel_size, ep=1,
                                   dp=strategy.data_parallel_size, pp=strategy.pipeline_model_parallel_size,
                                   cp=strategy.context_parallel_size, order=strategy.order)
        self.expert = RankGenerator(tp=strategy.expert_tensor_parallel_size,
                                    ep=strategy.expert_model_parallel_size,
                                    dp=strategy.expert_data_parallel_size,
                                    pp=strategy.pipeline_model_parallel_size, cp=1, order=strategy.order)
        if self.dense.get_ranks("pp") != self.expert.get_ranks("pp"):
            raise AssertionError("pipeline groups of the dense and expert meshes differ: "
                                 f"{self.dense.get_ranks('pp')} vs {self.expert.get_ranks('pp')}")

    def get_ranks(self, token: str, is_expert: bool = False) -> List[List[int]]:
        return (self.expert if is_expert else self.dense).get_ranks(token)
