"""Host validation of a transfer kernel's task table before it is launched.

The reshard kernel trusts its 64-byte tasks: absolute source / destination addresses, row and plane strides,
row and plane counts.  A wrong table writes into whatever memory the addresses name, so with
``EMB_VALIDATE_TASKS=1`` the native engine checks every new table first:

* the full footprint of every task (all planes, all rows) lies inside ONE source arena and ONE destination
  arena of the switch (a rank's parameter or ``[3, n]`` optimizer arena, sized from the plan);
* no byte is written by two tasks of the table (each destination byte has exactly one producer).

The reference has no equivalent: it issues one blocking NCCL call per (parameter, tensor, peer) and relies
on the call order (transfer/transfer.py:196-197).  This stands in for a sanitizer's bounds check on the
transfer where no memory sanitizer can run.
"""
from __future__ import annotations

import os
from typing import Dict, List, Sequence, Tuple

import numpy as np

Region = Tuple[int, int, str]  # (base address, bytes, label)


def enabled() -> bool:
    return os.environ.get("EMB_VALIDATE_TASKS", "0") not in ("", "0")


def plan_regions(plan, addrs: Dict[int, Sequence[int]], el_param: int) -> Tuple[List[Region], List[Region]]:
    """Source and destination arenas of a switch: ``addrs[r] = (src param, src opt, dst param, dst opt)``
    base addresses as seen by this process (0 = absent)."""
    src, dst = [], []
    for r, (sp, so, dp, do) in sorted(addrs.items()):
        if r < len(plan.src_param_numel):
            if sp:
                src.append((int(sp), plan.src_param_numel[r] * el_param, f"rank {r} source params"))
            if so:
                src.append((int(so), 3 * plan.src_opt_numel[r] * 4, f"rank {r} source optimizer"))
        if r < len(plan.dst_param_numel):
            if dp:
                dst.append((int(dp), plan.dst_param_numel[r] * el_param, f"rank {r} destination params"))
            if do:
                dst.append((int(do), 3 * plan.dst_opt_numel[r] * 4, f"rank {r} destination optimizer"))
    return src, dst


def _extent(t: np.ndarray, side: str) -> Tuple[np.ndarray, np.ndarray]:
    start = t[side].astype(np.int64)
    last = ((t["planes"].astype(np.int64) - 1) * t[side + "_plane"].astype(np.int64)
            + (t["rows"].astype(np.int64) - 1) * t[side + "_stride"].astype(np.int64))
    return start, start + last + t["row_bytes"].astype(np.int64)


def _inside(start: np.ndarray, end: np.ndarray, regions: List[Region]) -> np.ndarray:
    if not regions:
        return np.zeros(len(start), dtype=bool)
    reg = sorted(regions)
    bases = np.array([b for b, _, _ in reg], dtype=np.int64)
    ends = bases + np.array([n for _, n, _ in reg], dtype=np.int64)
    i = np.searchsorted(bases, start, side="right") - 1
    ok = i >= 0
    j = np.clip(i, 0, None)
    return ok & (start >= bases[j]) & (end <= ends[j])


def _row_intervals(t: np.ndarray, side: str) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Every (plane, row) byte interval of every task: (start, end, task index)."""
    rows = t["rows"].astype(np.int64)
    n = rows * t["planes"].astype(np.int64)
    idx = np.repeat(np.arange(len(t)), n)
    k = np.arange(int(n.sum())) - np.repeat(np.cumsum(n) - n, n)
    p, r = k // rows[idx], k % rows[idx]
    start = (t[side].astype(np.int64)[idx] + p * t[side + "_plane"].astype(np.int64)[idx]
             + r * t[side + "_stride"].astype(np.int64)[idx])
    return start, start + t["row_bytes"].astype(np.int64)[idx], idx


def validate_tasks(tasks: np.ndarray, src_regions: List[Region], dst_regions: List[Region],
                   check_overlap: bool = True, max_report: int = 5) -> None:
    """Raise ``ValueError`` naming the first offending tasks if the table breaks a rule above."""
    if len(tasks) == 0:
        return
    errors = []
    bad_rows = (tasks["rows"] == 0) | (tasks["row_bytes"] == 0) | (tasks["planes"] == 0)
    for i in np.flatnonzero(bad_rows)[:max_report]:
        errors.append(f"task {i}: empty (rows {tasks['rows'][i]}, row_bytes {tasks['row_bytes'][i]}, "
                      f"planes {tasks['planes'][i]})")
    for side, regions in (("src", src_regions), ("dst", dst_regions)):
        s, e = _extent(tasks, side)
        for i in np.flatnonzero(~_inside(s, e, regions))[:max_report]:
            errors.append(f"task {i}: {side} bytes [{s[i]:#x}, {e[i]:#x}) are not inside one "
                          f"{'source' if side == 'src' else 'destination'} arena")
    if check_overlap and not errors:
        s, e, idx = _row_intervals(tasks, "dst")
        o = np.argsort(s, kind="stable")
        s, e, idx = s[o], e[o], idx[o]
        reach = np.maximum.accumulate(e)
        clash = np.flatnonzero(s[1:] < reach[:-1]) + 1
        for k in clash[:max_report]:
            prev = int(np.flatnonzero(e[:k] > s[k])[-1])
            errors.append(f"tasks {idx[prev]} and {idx[k]} both write destination byte {s[k]:#x}")
    if errors:
        raise ValueError(f"{len(errors)} invalid transfer task(s):\n  " + "\n  ".join(errors))


# ---------------------------------------------------------------------------------------------------- checksums
_P1, _P2, _P3, _P4 = 0x9E3779B97F4A7C15, 0xC2B2AE3D27D4EB4F, 0x165667B19E3779F9, 0x27D4EB2F165667C5
_CHUNK = 1 << 22


def _wrap64(x: int) -> int:
    x &= (1 << 64) - 1
    return x - (1 << 64) if x >= 1 << 63 else x


def _piece_sum(arena, piece, tag: int) -> "torch.Tensor":
    """Sum over one piece of ``bits(value) * w(tag, global row, global col)`` in wrapping int64 arithmetic:
    exact and independent of summation order, so any layout of the same global state gives the same value."""
    import torch

    rows, cols = piece.gr1 - piece.gr0, piece.gc1 - piece.gc0
    ibits = torch.int16 if arena.element_size() == 2 else torch.int32
    dev = arena.device
    gc = torch.arange(piece.gc0, piece.gc1, device=dev, dtype=torch.int64) * _wrap64(_P2)
    total = torch.zeros((), dtype=torch.int64, device=dev)
    step = max(1, _CHUNK // max(cols, 1))
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        blk = arena.as_strided((r1 - r0, cols), (piece.ld, 1), piece.off(piece.gr0 + r0, piece.gc0))
        b = blk.view(ibits).to(torch.int64)
        gr = torch.arange(piece.gr0 + r0, piece.gr0 + r1, device=dev, dtype=torch.int64) * _wrap64(_P1)
        w = gr[:, None] + gc[None, :] + _wrap64(tag * _P3)
        w = (w ^ (w >> 31)) * _wrap64(_P4)
        w = w ^ (w >> 29)
        total += (b * (w | 1)).sum()
    return total


def state_checksum(ts, group=None) -> Tuple[int, int]:
    """Layout-independent, position-sensitive checksums ``(params, optimizer state)`` of the whole model state
    of ``ts``'s strategy (a collective over its ranks when ``group`` is given).

    Every global element of every parameter is counted once: from the lowest rank of its first pipeline stage
    that holds its TP piece, and its fp32 master / exp_avg / exp_avg_sq from the optimizer-instance-0 rank that
    owns it.  The bits of each value are weighted by a hash of (parameter, plane, global row, global column) and
    summed with int64 wrap-around, so two strategies holding the same state bit for bit give equal checksums,
    and a value moved to the wrong place or changed in any bit changes them.  Used after timed switches to
    check the moved bytes against the planner's index maps (the oracle)."""
    import torch
    import torch.distributed as dist

    from ..config import get_args
    from ..models.spec import stages_of
    from ..planner.layout import virtual_params
    from ..planner.plan import _StrategyView

    args = get_args()
    cfg, tc = args.model, args.train
    s, r = ts.strategy, ts.rank
    view = _StrategyView(cfg, s, tc.overlap_grad_reduce, tc.ddp_bucket_size)
    zc = [s.zero_coords(q) for q in range(s.world_size)]
    P, O = ts.param_flat, ts.opt_flat
    acc_p = torch.zeros((), dtype=torch.int64, device=P.device)
    acc_o = torch.zeros((), dtype=torch.int64, device=P.device)
    for vp in virtual_params(cfg):
        hold = view.holders(vp)
        if r not in hold:
            continue
        first = min(stages_of(vp, cfg, s.pipeline_model_parallel_size))
        if view.coords[r]["pp"] != first:
            continue
        tkey = lambda q: (view.coords[q]["etp"] if vp.is_expert else view.coords[q]["tp"]) if vp.tp_dim is not None else 0
        mine = tkey(r)
        if min(q for q in hold if view.coords[q]["pp"] == first and tkey(q) == mine) == r:
            for pc in view.param_pieces(vp, r):
                acc_p += _piece_sum(P, pc, 4 * vp.index)
        # optimizer state: one owner per (TP piece, ZeRO shard) among instance-0 ranks (TP-replicated parameters
        # keep a copy of their sharded state on every TP rank)
        def okey(q):
            zq = zc[q]
            inst = zq["expert_instance"] if vp.is_expert else zq["dense_instance"]
            return (tkey(q), zq["expert_shard"] if vp.is_expert else zq["dense_shard"]) if inst == 0 else None

        if okey(r) is not None and min(q for q in hold if view.coords[q]["pp"] == first and okey(q) == okey(r)) == r:
            for pc in view.opt_pieces(vp, r):
                for plane in range(3):
                    acc_o += _piece_sum(O[plane], pc, 4 * vp.index + 1 + plane)
    out = torch.stack([acc_p, acc_o])
    if group is not None and dist.is_initialized():
        if dist.get_backend(group) == "nccl" and out.device.type != "cuda":
            out = out.cuda()
        dist.all_reduce(out, group=group)
    a, b = out.tolist()
    return int(a), int(b)
