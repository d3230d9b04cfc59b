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
