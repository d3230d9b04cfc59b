"""Heterogeneous data parallelism: uneven micro-batch counts per DP rank.

When ``global_batch_size`` is not divisible by ``micro_batch_size * DP`` (for example after scaling to a
world size that does not divide the batch), the reference patches Megatron's micro-batch calculator and
forward step so that DP ranks run different numbers of micro-batches and the per-micro-batch losses are
padded and all-reduced afterwards (elastic_megatron/hetero_dp.py:126-256).

Here the pieces are native to the training core:

* ``runtime/data.py``: ``num_microbatches(..., hetero=True)`` gives the first ``units % DP`` ranks one extra
  unit of ``alignment`` micro-batches and the sampler deals the units of a global batch round-robin over DP
  ranks, so the set of samples per global batch does not depend on DP;
* ``runtime/train.py``: the loss scale is uniform (``DP*CP / (GBS*seq)``) and the loss report is one sum
  all-reduce, so no padding of per-micro-batch losses is needed;
* gradient reduction, pipeline schedules and the optimizer are unchanged (all stages of one pipeline share a
  DP rank, hence a micro-batch count).

:func:`apply_hetero_dp` switches the mode on for every subsequent ``train_step``; it takes the reference's
arguments (elastic_megatron/hetero_dp.py:191): ``alignment`` makes every DP rank's micro-batch count a
multiple of it (units of ``alignment`` micro-batches are dealt over the DP ranks, the first ranks taking the
remainder), and ``process_fwd_bwd_outputs`` is an optional hook on the per-micro-batch outputs.  The reference
needs that hook to pad Megatron's per-micro-batch loss dicts to the DP maximum and all-reduce them
(hetero_dp.py:62-123); the loss report here needs none, so by default the outputs pass through unchanged.
"""
from __future__ import annotations

from typing import Callable, List, Optional

_ENABLED = False
_ALIGNMENT = 1
_PROCESS: Optional[Callable] = None


def apply_hetero_dp(process_fwd_bwd_outputs: Optional[Callable] = None, alignment: int = 1,
                    enabled: bool = True) -> None:
    """Enable (or with ``enabled=False`` disable) uneven micro-batch counts over DP ranks.

    ``process_fwd_bwd_outputs(outputs)`` is called on the last pipeline stage with this rank's list of
    per-micro-batch token-loss sums (one scalar tensor each) and returns the list that the loss report sums.
    """
    global _ENABLED, _ALIGNMENT, _PROCESS
    if process_fwd_bwd_outputs is not None and not callable(process_fwd_bwd_outputs):
        raise TypeError("process_fwd_bwd_outputs must be callable (use enabled=False to switch hetero-DP off)")
    if int(alignment) < 1:
        raise ValueError(f"alignment must be >= 1, got {alignment}")
    _ENABLED = bool(enabled)
    _ALIGNMENT = int(alignment)
    _PROCESS = process_fwd_bwd_outputs


def hetero_dp_enabled() -> bool:
    return _ENABLED


def hetero_alignment() -> int:
    return _ALIGNMENT if _ENABLED else 1


def process_outputs(outputs: List) -> List:
    return _PROCESS(outputs) if (_ENABLED and _PROCESS is not None) else outputs
