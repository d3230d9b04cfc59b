"""Convert a checkpoint to another parallel strategy offline, optionally comparing against a reference.

    python -m elasticmegatron_b200.tools.convert_ckpt before_reshard converted --tp 2 --pp 1 --world-size 2 \
        --compare after_reshard

The reference does this with Megatron's ``tools/checkpoint/convert.py`` behind a loader patched to force the
source TP/PP/EP (tools/ckpt/run_convert_patch_loader.py:27-133), then compares the result with the checkpoint
written right after an online reshard (tools/ckpt/convert_and_compare.sh:31-70).  Here the source layout is
read from the checkpoint itself (every rank file records its strategy), the conversion goes through the same
layout-free global tensors as ``load_checkpoint`` (``runtime/checkpoint.py``), and ``--compare`` runs
``compare_ckpt`` on the result.  One process, CPU only, no process groups.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch


def _saved_args(root: str, iteration):
    from ..config import Args, ModelConfig, TrainConfig
    from ..runtime.checkpoint import read_latest

    if iteration is None:
        iteration = read_latest(root)
    it_dir = os.path.join(root, f"iter_{iteration:07d}")
    first = next(os.path.join(it_dir, sub, "model_optim_rng.pt") for sub in sorted(os.listdir(it_dir))
                 if os.path.exists(os.path.join(it_dir, sub, "model_optim_rng.pt")))
    meta = torch.load(first, weights_only=False)
    a = meta["args"]
    return Args(model=ModelConfig(**a["model"]), train=TrainConfig(**a["train"])), iteration


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--iteration", type=int, default=None)
    ap.add_argument("--world-size", type=int, required=True)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--cp", type=int, default=1)
    ap.add_argument("--ep", type=int, default=1)
    ap.add_argument("--instances", type=int, default=1, help="Group-ZeRO distributed-optimizer instances")
    ap.add_argument("--compare", default=None, help="checkpoint root to compare the converted one against")
    ap.add_argument("--thresh", type=float, default=1e-3)
    a = ap.parse_args(argv)

    from ..config import set_args
    from ..parallel.strategy import ParallelStrategy
    from ..runtime.checkpoint import convert_checkpoint

    args, it = _saved_args(a.src, a.iteration)
    set_args(args)
    dst = ParallelStrategy(world_size=a.world_size, tensor_model_parallel_size=a.tp,
                           pipeline_model_parallel_size=a.pp, context_parallel_size=a.cp,
                           expert_model_parallel_size=a.ep, num_distributed_optimizer_instances=a.instances)
    convert_checkpoint(a.src, a.dst, dst, it)
    print(f"converted {a.src} iteration {it} -> {a.dst} as {dst}")
    if a.compare:
        from .compare_ckpt import main as compare_main

        return compare_main([os.path.join(a.dst, f"iter_{it:07d}"), os.path.join(a.compare, f"iter_{it:07d}"),
                             "--thresh", str(a.thresh)])
    return 0


if __name__ == "__main__":
    sys.exit(main())
