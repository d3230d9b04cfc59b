"""Heterogeneous data parallelism: uneven micro-batch counts per DP rank.

When ``global_batch_size`` is not divisible by ``micro_batch_size * DP`` (for example after scaling to a
world size that does not divide the batch), the reference patches Megatron's micro-batch calculator and
forward step so that DP ranks run different numbers of micro-batches and the per-micro-batch losses are
padded and all-reduced afterwards (elastic_megatron/hetero_dp.py:126-256).

Here the pieces are native to the training core:

* ``runtime/data.py``: ``num_microbatches(..., hetero=True)`` gives the first ``n_mb % DP`` ranks one extra
  micro-batch and the sampler deals the micro-batches of a global batch round-robin over DP ranks, so the
  set of samples per global batch does not depend on DP;
* ``runtime/train.py``: the loss scale is uniform (``DP*CP / (GBS*seq)``) and the loss report is one sum
  all-reduce, so no padding of per-micro-batch losses is needed;
* gradient reduction, pipeline schedules and the optimizer are unchanged (all stages of one pipeline share a
  DP rank, hence a micro-batch count).

:func:`apply_hetero_dp` switches the mode on for every subsequent ``train_step`` (the reference's entry point
has the same name).
"""
from __future__ import annotations

_ENABLED = False


def apply_hetero_dp(enabled: bool = True) -> None:
    global _ENABLED
    _ENABLED = bool(enabled)


def hetero_dp_enabled() -> bool:
    return _ENABLED
