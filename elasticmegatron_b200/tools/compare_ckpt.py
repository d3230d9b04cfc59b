"""Compare two checkpoints tensor by tensor (model weights), the check the reference runs after a reshard.

    python -m elasticmegatron_b200.tools.compare_ckpt A/iter_0000010 B/iter_0000010 --thresh 1e-3

Every ``<subdir>/model_optim_rng.pt`` present under both roots is loaded and its ``model`` dict compared: the
key sets must match, shapes must match, and the relative RMS difference ``||a - b|| / ||a||`` of each tensor
must not exceed ``--thresh`` (default 1e-3, as in the reference's tools/ckpt/compare_ckpt.py).  Exit code 1
when anything differs.
"""
from __future__ import annotations

import argparse
import os
import sys
from typing import Dict, List, Tuple

import torch


def _files(root: str) -> Dict[str, str]:
    out = {}
    for dirpath, _, files in os.walk(root):
        if "model_optim_rng.pt" in files:
            out[os.path.relpath(dirpath, root)] = os.path.join(dirpath, "model_optim_rng.pt")
    return out


def rel_rms(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    den = a.pow(2).mean().sqrt().item()
    num = (a - b).pow(2).mean().sqrt().item()
    return num / den if den > 0 else num


def compare(root_a: str, root_b: str, thresh: float = 1e-3) -> List[Tuple[str, str, str]]:
    """Returns a list of (file, tensor, problem); empty when the checkpoints agree."""
    fa, fb = _files(root_a), _files(root_b)
    problems = []
    for rel in sorted(set(fa) | set(fb)):
        if rel not in fa or rel not in fb:
            problems.append((rel, "*", "missing in " + ("A" if rel not in fa else "B")))
            continue
        ma = torch.load(fa[rel], weights_only=False)["model"]
        mb = torch.load(fb[rel], weights_only=False)["model"]
        for k in sorted(set(ma) | set(mb)):
            if k not in ma or k not in mb:
                problems.append((rel, k, "missing key"))
            elif tuple(ma[k].shape) != tuple(mb[k].shape):
                problems.append((rel, k, f"shape {tuple(ma[k].shape)} vs {tuple(mb[k].shape)}"))
            else:
                e = rel_rms(ma[k], mb[k])
                if e > thresh:
                    problems.append((rel, k, f"rel-rms {e:.3e} > {thresh:g}"))
    return problems


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("a")
    ap.add_argument("b")
    ap.add_argument("--thresh", type=float, default=1e-3)
    a = ap.parse_args(argv)
    probs = compare(a.a, a.b, a.thresh)
    for p in probs:
        print(" | ".join(p))
    print("MATCH" if not probs else f"{len(probs)} mismatches")
    return 0 if not probs else 1


if __name__ == "__main__":
    sys.exit(main())
