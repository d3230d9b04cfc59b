"""Extract loss / step-time curves from training logs (the reference plots them; here: CSV + a text summary).

    python -m elasticmegatron_b200.tools.loss_curve run_a.log run_b.log --csv curves.csv

Understands this framework's JSON lines (``{"event": "iteration", "iteration": i, "loss": x, "ms": t, ...}``),
Megatron-style text lines (``iteration   10/ ... lm loss: 1.2E+01 ... elapsed time per iteration (ms): 123``)
and plain files with one loss per line.  With several logs, the report gives the maximum relative loss
difference against the first log at every common iteration (the loss-continuity check after a switch).
"""
from __future__ import annotations

import argparse
import csv
import json
import re
import sys
from typing import Dict, List, Tuple

_ITER = re.compile(r"iteration\s+(\d+)\s*/")
_LOSS = re.compile(r"lm loss:\s*([0-9.eE+-]+)")
_TIME = re.compile(r"elapsed time per iteration \(ms\):\s*([0-9.eE+-]+)")


def read_log(path: str) -> Dict[int, Tuple[float, float]]:
    """{iteration: (loss, ms)}"""
    out: Dict[int, Tuple[float, float]] = {}
    plain: List[float] = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                try:
                    d = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if d.get("event") == "iteration" and "loss" in d:
                    out[int(d["iteration"])] = (float(d["loss"]), float(d.get("ms", "nan")))
                continue
            m = _ITER.search(line)
            l = _LOSS.search(line)
            if m and l:
                t = _TIME.search(line)
                out[int(m.group(1))] = (float(l.group(1)), float(t.group(1)) if t else float("nan"))
                continue
            try:
                plain.append(float(line))
            except ValueError:
                pass
    if not out and plain:
        out = {i + 1: (v, float("nan")) for i, v in enumerate(plain)}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("logs", nargs="+")
    ap.add_argument("--csv", default=None)
    a = ap.parse_args(argv)
    curves = [read_log(p) for p in a.logs]
    if a.csv:
        its = sorted(set().union(*[set(c) for c in curves]))
        with open(a.csv, "w", newline="") as f:
            w = csv.writer(f)
            w.writerow(["iteration"] + [f"loss_{i}" for i in range(len(curves))] + [f"ms_{i}" for i in range(len(curves))])
            for it in its:
                w.writerow([it] + [c.get(it, (None, None))[0] for c in curves] + [c.get(it, (None, None))[1] for c in curves])
    base = curves[0]
    for p, c in zip(a.logs, curves):
        common = sorted(set(base) & set(c))
        worst = max((abs(c[i][0] - base[i][0]) / abs(base[i][0]) for i in common if base[i][0]), default=0.0)
        print(f"{p}: {len(c)} iterations, last loss {c[max(c)][0] if c else float('nan'):.4f}, "
              f"max rel diff vs first log {worst:.2e}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
