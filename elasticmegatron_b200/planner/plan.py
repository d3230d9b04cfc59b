"""Exact-range reshard planner.

Given a source and a destination strategy, produce the list of 2-D copies that turn every rank's source
state into its destination state:

* ``KIND_OPT``   - fp32 optimizer state (master weight, ``exp_avg``, ``exp_avg_sq``): three planes of one
  ``[3, n]`` optimizer arena, copied with identical offsets;
* ``KIND_PARAM`` - the model parameter (bf16 on GPU, fp32 in CPU runs) for the *whole* destination TP shard.
  Parameters are replicated over DP/CP and always equal ``cast(master)``, so the destination pulls them
  from the nearest source replica instead of regenerating them from the master and all-gathering.

The reference plans in three phases per parameter - gather every ZeRO shard on an "aligned" rank, move TP
chunks between aligned ranks, scatter into the destination ZeRO shards (elastic_megatron/transfer/
transfer.py:143-269; plan construction resharding/resharding.py:48-156, resharding_tp.py:94-191) - with
padded full tensors and SwiGLU shuffle copies in between.  This planner instead intersects, in the global
(TP=1) coordinates of each virtual parameter, every piece a source rank holds with every piece a destination
rank needs; each non-empty intersection is one strided copy directly from the source arena to the
destination arena.  SwiGLU halves, GQA group order, vocab padding and expert homes are index maps
(``models/spec.py``), so no intermediate tensors exist.

A *piece* is a 2-D box of one rank's local TP shard of a virtual parameter that is contiguous in the rank's
arena: a 1-D ZeRO range over an ``[R, C]`` shard splits into at most three boxes (partial first row, full
rows, partial last row), and a box splits further where the TP row map (SwiGLU) is discontinuous.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from ..config import ModelConfig, get_args
from ..models.spec import VParam, stages_of, tp_col_offset, tp_row_blocks
from .layout import RankLayout, rank_layout, virtual_params

KIND_OPT = 0
KIND_PARAM = 1

DESC_DTYPE = np.dtype([
    ("src_rank", np.int32), ("dst_rank", np.int32), ("kind", np.int32), ("vp", np.int32),
    ("src_off", np.int64), ("dst_off", np.int64), ("rows", np.int64), ("cols", np.int64),
    ("src_stride", np.int64), ("dst_stride", np.int64),
])


@dataclass
class _Piece:
    gr0: int
    gr1: int
    gc0: int
    gc1: int
    row_delta: int  # local_row = global_row + row_delta
    col_delta: int  # local_col = global_col + col_delta
    base: int  # arena offset of local flat index 0
    ld: int  # local row length

    def off(self, gr: int, gc: int) -> int:
        return self.base + (gr + self.row_delta) * self.ld + (gc + self.col_delta)


def _as2d(shape: Tuple[int, ...]) -> Tuple[int, int]:
    if len(shape) == 1:
        return 1, shape[0]
    r = 1
    for s in shape[:-1]:
        r *= s
    return r, shape[-1]


def _flat_to_boxes(f0: int, f1: int, C: int) -> List[Tuple[int, int, int, int]]:
    """Split local flat range [f0, f1) of a row-major [*, C] matrix into boxes (r0, r1, c0, c1)."""
    if f0 >= f1:
        return []
    r0, c0 = divmod(f0, C)
    r1, c1 = divmod(f1 - 1, C)
    c1 += 1
    if r0 == r1:
        return [(r0, r0 + 1, c0, c1)]
    out = []
    mid0, mid1 = r0, r1 + 1
    if c0 > 0:
        out.append((r0, r0 + 1, c0, C))
        mid0 = r0 + 1
    if c1 < C:
        mid1 = r1
    if mid1 > mid0:
        out.append((mid0, mid1, 0, C))
    if c1 < C:
        out.append((r1, r1 + 1, 0, c1))
    return out


def _pieces(vp: VParam, tp: int, tp_rank: int, local_shape, flat_ranges, base_of_range) -> List[_Piece]:
    """Global pieces of local flat ranges of ``vp``'s TP shard.

    ``flat_ranges`` are (f0, f1) local flat ranges, ``base_of_range[i]`` the arena offset of local flat 0
    valid inside range ``i``.
    """
    R, C = _as2d(local_shape)
    if vp.tp_dim == 0 or vp.tp_dim is None:
        blocks = tp_row_blocks(vp, tp, tp_rank) if vp.tp_dim == 0 else [(0, 0, R)]
        coff = 0
    else:
        blocks = [(0, 0, R)]
        coff = tp_col_offset(vp, tp, tp_rank)
    out = []
    for (f0, f1), base in zip(flat_ranges, base_of_range):
        for (lr0, lr1, c0, c1) in _flat_to_boxes(f0, f1, C):
            for (g0, l0, n) in blocks:
                a, b = max(lr0, l0), min(lr1, l0 + n)
                if a >= b:
                    continue
                delta = l0 - g0
                out.append(_Piece(a - delta, b - delta, c0 + coff, c1 + coff, delta, -coff, base, C))
    return out


def _intersect(s: _Piece, d: _Piece):
    r0, r1 = max(s.gr0, d.gr0), min(s.gr1, d.gr1)
    if r0 >= r1:
        return None
    c0, c1 = max(s.gc0, d.gc0), min(s.gc1, d.gc1)
    if c0 >= c1:
        return None
    return r0, r1, c0, c1


class _StrategyView:
    """Holders of each virtual parameter under one strategy, with their pieces."""

    def __init__(self, cfg: ModelConfig, strategy, overlap: bool, bucket: Optional[int]):
        self.cfg, self.s = cfg, strategy
        self.layouts: List[RankLayout] = [rank_layout(cfg, strategy, r, overlap, bucket)
                                          for r in range(strategy.world_size)]
        self.coords = [strategy.coords(r) for r in range(strategy.world_size)]

    def holders(self, vp: VParam) -> List[int]:
        st = stages_of(vp, self.cfg, self.s.pipeline_model_parallel_size)
        out = []
        for r, c in enumerate(self.coords):
            if c["pp"] not in st:
                continue
            if vp.is_expert and vp.expert_id // self.s.expert_num_per_ep_rank != c["ep"]:
                continue
            out.append(r)
        return out

    def tp_of(self, vp: VParam, r: int) -> Tuple[int, int]:
        if vp.is_expert:
            return self.s.expert_tensor_parallel_size, self.coords[r]["etp"]
        return self.s.tensor_model_parallel_size, self.coords[r]["tp"]

    def param_pieces(self, vp: VParam, r: int) -> List[_Piece]:
        P, shp = self.layouts[r].vp_loc[vp.index]
        n = 1
        for x in shp:
            n *= x
        tp, t = self.tp_of(vp, r)
        return _pieces(vp, tp, t, shp, [(0, n)], [P])

    def opt_pieces(self, vp: VParam, r: int) -> List[_Piece]:
        rl = self.layouts[r]
        P, shp = rl.vp_loc[vp.index]
        n = 1
        for x in shp:
            n *= x
        ranges, bases = [], []
        for s, e, o in rl.owned_overlapping(P, P + n):
            lo, hi = max(s, P), min(e, P + n)
            if lo < hi:
                ranges.append((lo - P, hi - P))
                bases.append(o + P - s)
        tp, t = self.tp_of(vp, r)
        return _pieces(vp, tp, t, shp, ranges, bases)

    def replica_key(self, vp: VParam, r: int, kind: int):
        """Ranks with equal keys hold identical data of ``vp`` at identical offsets (the stage is part of the
        key: the two copies of a tied embedding sit at different offsets of different layouts)."""
        c = self.coords[r]
        # a TP-replicated parameter (tp_dim None) is identical on every TP rank
        t = (c["etp"] if vp.is_expert else c["tp"]) if vp.tp_dim is not None else 0
        if kind == KIND_PARAM:
            return (c["pp"], t)
        rl = self.layouts[r]
        z = rl.expert_shard_index if vp.is_expert else rl.dense_shard_index
        return (c["pp"], t, z)


@dataclass
class ReshardPlan:
    src: object
    dst: object
    desc: np.ndarray  # DESC_DTYPE records
    src_opt_numel: List[int]
    dst_opt_numel: List[int]
    src_param_numel: List[int]
    dst_param_numel: List[int]

    def for_rank(self, rank: int, role: str = "dst") -> np.ndarray:
        key = "dst_rank" if role == "dst" else "src_rank"
        return self.desc[self.desc[key] == rank]

    def bytes_matrix(self, opt_elem: int = 4, param_elem: int = 2, n: Optional[int] = None) -> np.ndarray:
        """[src, dst] bytes moved (opt counts its three planes)."""
        n = n or max(self.src.world_size, self.dst.world_size)
        m = np.zeros((n, n), dtype=np.int64)
        el = self.desc["rows"] * self.desc["cols"]
        by = np.where(self.desc["kind"] == KIND_OPT, el * 3 * opt_elem, el * param_elem)
        np.add.at(m, (self.desc["src_rank"], self.desc["dst_rank"]), by)
        return m

    def describe(self, cfg: Optional[ModelConfig] = None, ranks: Optional[Iterable[int]] = None,
                 max_params: Optional[int] = None) -> str:
        """Human-readable plan: per virtual parameter, which ranks send how many elements of which state to
        which ranks (the reference prints the same per-parameter send / receive plan in its debug mode,
        transfer/transfer.py:271-289).  ``ranks`` restricts it to copies that touch those ranks."""
        cfg = cfg or get_args().model
        names = {vp.index: vp.name for vp in virtual_params(cfg)}
        d = self.desc
        if ranks is not None:
            rs = np.array(sorted(set(ranks)))
            d = d[np.isin(d["src_rank"], rs) | np.isin(d["dst_rank"], rs)]
        lines = [f"reshard plan {self.src} -> {self.dst}: {len(d)} copies"]
        vps = np.unique(d["vp"])
        for i, v in enumerate(vps):
            if max_params is not None and i >= max_params:
                lines.append(f"  ... {len(vps) - max_params} more parameters")
                break
            dv = d[d["vp"] == v]
            lines.append(f"  {names.get(int(v), v)}")
            for kind, label in ((KIND_OPT, "fp32 master+moments"), (KIND_PARAM, "bf16 param")):
                dk = dv[dv["kind"] == kind]
                if not len(dk):
                    continue
                pairs = {}
                for row in dk:
                    key = (int(row["src_rank"]), int(row["dst_rank"]))
                    pairs[key] = pairs.get(key, 0) + int(row["rows"]) * int(row["cols"])
                moves = ", ".join(f"{s}->{t}:{n}" for (s, t), n in sorted(pairs.items()))
                lines.append(f"    {label}: {moves}")
        return "\n".join(lines)

    def nvlink_roofline_ms(self, link_gbs: float, opt_elem: int = 4, param_elem: int = 2) -> float:
        """max over GPUs of max(egress, ingress) of non-local bytes / link bandwidth."""
        m = self.bytes_matrix(opt_elem, param_elem)
        np.fill_diagonal(m, 0)
        worst = max(m.sum(0).max(initial=0), m.sum(1).max(initial=0))
        return worst / (link_gbs * 1e9) * 1e3


def _choose(cands: Sequence[int], dst_rank: int, salt: int) -> int:
    if dst_rank in cands:
        return dst_rank
    return cands[(dst_rank + salt) % len(cands)]


def _merge_rows(rows, cols, sst, dstd):
    if rows > 1 and cols == sst and cols == dstd:
        return 1, rows * cols
    return rows, cols


def build_plan(src, dst, cfg: Optional[ModelConfig] = None, kinds: Iterable[int] = (KIND_OPT, KIND_PARAM),
               overlap_grad_reduce: Optional[bool] = None, ddp_bucket_size: Optional[int] = None,
               allowed_src: Optional[Iterable[int]] = None) -> ReshardPlan:
    """Plan the switch ``src -> dst``.

    ``allowed_src`` restricts which source ranks may be read (failure recovery: only survivors); a piece of
    state with no allowed holder raises ``RuntimeError`` (the state is lost without a Group-ZeRO replica).
    """
    args = get_args()
    cfg = cfg or args.model
    if overlap_grad_reduce is None:
        overlap_grad_reduce = args.train.overlap_grad_reduce
        ddp_bucket_size = args.train.ddp_bucket_size
    allowed = set(allowed_src) if allowed_src is not None else None
    sv = _StrategyView(cfg, src, overlap_grad_reduce, ddp_bucket_size)
    dv = _StrategyView(cfg, dst, overlap_grad_reduce, ddp_bucket_size)
    recs = []
    for vp in virtual_params(cfg):
        sh, dh = sv.holders(vp), dv.holders(vp)
        for kind in kinds:
            # source replica classes
            classes: Dict[tuple, List[int]] = {}
            for r in sh:
                classes.setdefault(sv.replica_key(vp, r, kind), []).append(r)
            src_pieces = []
            for key, members in classes.items():
                rep = members[0]
                pcs = sv.param_pieces(vp, rep) if kind == KIND_PARAM else sv.opt_pieces(vp, rep)
                src_pieces.append((members, pcs))
            dcache: Dict[tuple, List[_Piece]] = {}
            for d in dh:
                dkey = dv.replica_key(vp, d, kind)
                dp = dcache.get(dkey)
                if dp is None:
                    dp = dv.param_pieces(vp, d) if kind == KIND_PARAM else dv.opt_pieces(vp, d)
                    dcache[dkey] = dp
                for members, spcs in src_pieces:
                    cands = members if allowed is None else [m for m in members if m in allowed]
                    if not cands:
                        raise RuntimeError(f"no surviving source holds {vp.name} (kind {kind}) for rank {d}")
                    srank = _choose(cands, d, vp.index)
                    for sp in spcs:
                        for dpp in dp:
                            box = _intersect(sp, dpp)
                            if box is None:
                                continue
                            r0, r1, c0, c1 = box
                            rows, cols = _merge_rows(r1 - r0, c1 - c0, sp.ld, dpp.ld)
                            recs.append((srank, d, kind, vp.index, sp.off(r0, c0), dpp.off(r0, c0), rows, cols,
                                         sp.ld, dpp.ld))
    desc = np.array(recs, dtype=DESC_DTYPE) if recs else np.zeros(0, dtype=DESC_DTYPE)
    return ReshardPlan(src=src, dst=dst, desc=desc,
                       src_opt_numel=[l.opt_numel for l in sv.layouts],
                       dst_opt_numel=[l.opt_numel for l in dv.layouts],
                       src_param_numel=[l.param_numel for l in sv.layouts],
                       dst_param_numel=[l.param_numel for l in dv.layouts])


def apply_plan_reference(plan: ReshardPlan, src_opt: Dict[int, "np.ndarray"], src_param: Dict[int, "np.ndarray"],
                         dst_opt: Dict[int, "np.ndarray"], dst_param: Dict[int, "np.ndarray"]) -> None:
    """Execute a plan on host arrays (the CPU oracle for every transfer engine).

    ``*_opt[r]`` are ``[3, n]`` arrays, ``*_param[r]`` flat arrays, indexed by rank.
    """
    for d in plan.desc:
        rows, cols = int(d["rows"]), int(d["cols"])
        so, do, ss, ds = int(d["src_off"]), int(d["dst_off"]), int(d["src_stride"]), int(d["dst_stride"])
        s, t = int(d["src_rank"]), int(d["dst_rank"])
        if d["kind"] == KIND_OPT:
            S, D = src_opt[s], dst_opt[t]
            for i in range(rows):
                D[:, do + i * ds: do + i * ds + cols] = S[:, so + i * ss: so + i * ss + cols]
        else:
            S, D = src_param[s], dst_param[t]
            for i in range(rows):
                D[do + i * ds: do + i * ds + cols] = S[so + i * ss: so + i * ss + cols]
