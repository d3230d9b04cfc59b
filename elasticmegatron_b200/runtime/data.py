"""Synthetic GPT data, a resumable DP sampler and the micro-batch calculator.

* :class:`MockGPTDataset` - sample ``i`` is ``seq_len + 1`` uniform token ids drawn from a generator seeded
  by ``(seed, i)``: any rank can produce any sample, so data is layout-independent (Megatron ``--mock-data``,
  run_e2e_demo.sh:149-161).
* :class:`PretrainingSampler` - the global batch at ``consumed_samples`` is the next ``GBS`` sample indices;
  DP rank ``r`` takes micro-batch ``[r*mbs, (r+1)*mbs)`` of each ``mbs*DP`` slice, so the set of samples per
  global batch is the same under every DP size (data continuity across switches; reference
  dataloader_state.py:127-157 resumes from ``consumed_train_samples`` the same way).
* :func:`num_microbatches` - ``GBS / (MBS * DP)``, reconfigured on every switch; hetero-DP gives the
  remainder, in units of ``alignment`` micro-batches, to the lowest DP ranks
  (elastic_megatron/hetero_dp.py:126-188).
* The iterator yields micro-batches in **pinned host memory**; the train step copies each to the device
  with ``non_blocking=True`` (the end-to-end path).
"""
from __future__ import annotations

from typing import Callable, Iterator, List, Optional, Tuple

import torch


class MockGPTDataset:
    def __init__(self, num_samples: int, seq_length: int, vocab_size: int, seed: int = 0):
        self.num_samples, self.seq_length, self.vocab_size, self.seed = num_samples, seq_length, vocab_size, seed

    def __len__(self):
        return self.num_samples

    def __getitem__(self, i: int) -> torch.Tensor:
        g = torch.Generator().manual_seed(self.seed * 1_000_000_007 + int(i))
        return torch.randint(0, self.vocab_size, (self.seq_length + 1,), generator=g, dtype=torch.int64)


def num_microbatches(global_batch_size: int, micro_batch_size: int, dp: int, dp_rank: int = 0,
                     hetero: bool = False, alignment: int = 1) -> int:
    per = micro_batch_size * dp
    if global_batch_size % per == 0:
        return global_batch_size // per
    if not hetero:
        raise ValueError(f"global batch {global_batch_size} not divisible by micro batch {micro_batch_size} x DP {dp}"
                         " (enable hetero-DP)")
    total_mb = global_batch_size // micro_batch_size
    if total_mb * micro_batch_size != global_batch_size or total_mb % alignment:
        raise ValueError(f"global batch {global_batch_size} must divide by micro batch {micro_batch_size} x "
                         f"alignment {alignment}")
    units = total_mb // alignment
    if units < dp:
        raise ValueError(f"{units} units of {alignment} micro-batches cannot feed {dp} DP ranks")
    base, extra = divmod(units, dp)
    return (base + (1 if dp_rank < extra else 0)) * alignment


class PretrainingSampler:
    """Sample indices for one DP rank, micro-batch by micro-batch, from ``consumed_samples`` on."""

    def __init__(self, total_samples: int, consumed_samples: int, micro_batch_size: int, dp_rank: int,
                 dp_size: int, global_batch_size: Optional[int] = None, alignment: int = 1):
        self.total, self.consumed = total_samples, consumed_samples
        self.mbs, self.r, self.dp = micro_batch_size, dp_rank, dp_size
        self.gbs = global_batch_size
        self.alignment = alignment

    def __iter__(self) -> Iterator[List[int]]:
        i = self.consumed
        while True:
            if self.gbs is None or self.gbs % (self.mbs * self.dp) == 0:
                s = i + self.r * self.mbs
                yield [(s + j) % self.total for j in range(self.mbs)]
                i += self.mbs * self.dp
            else:
                # hetero-DP: units of ``alignment`` micro-batches of one global batch are dealt round-robin
                # over DP ranks
                n_mb = self.gbs // self.mbs
                for m in range(n_mb):
                    if (m // self.alignment) % self.dp == self.r:
                        s = i + m * self.mbs
                        yield [(s + j) % self.total for j in range(self.mbs)]
                i += self.gbs


class DataIterator:
    """Yields (ids, labels) micro-batches ``[mbs, seq_local]`` in pinned host memory for one rank."""

    def __init__(self, dataset: MockGPTDataset, sampler: PretrainingSampler, positions: Optional[torch.Tensor],
                 pin: bool = True):
        self.ds, self.sampler, self.pos = dataset, sampler, positions
        self._it = iter(sampler)
        self.pin = pin and torch.cuda.is_available()

    def __iter__(self):
        return self

    def __next__(self) -> Tuple[torch.Tensor, torch.Tensor]:
        idx = next(self._it)
        toks = torch.stack([self.ds[i] for i in idx])
        ids, labels = toks[:, :-1], toks[:, 1:]
        if self.pos is not None:
            ids, labels = ids[:, self.pos], labels[:, self.pos]
        ids, labels = ids.contiguous(), labels.contiguous()
        if self.pin:
            ids, labels = ids.pin_memory(), labels.pin_memory()
        return ids, labels


class DataloaderState:
    """Dataset cache + iterator rebuild on every switch (reference: megatron_manager/dataloader_state.py)."""

    train_valid_test_datasets_provider: Optional[Callable] = None
    datasets = None
    _mock_key = None  # (seq_length, vocab_size, seed) of the cached mock datasets

    @classmethod
    def register(cls, provider: Callable) -> None:
        cls.train_valid_test_datasets_provider = provider
        cls.datasets = None

    @classmethod
    def get_datasets(cls, model_cfg, seed: int):
        """Registered datasets are built once; the synthetic ones are rebuilt when the model's sequence length,
        vocabulary or the seed changes (a new model in the same process)."""
        if cls.train_valid_test_datasets_provider is not None:
            if cls.datasets is None:
                cls.datasets = cls.train_valid_test_datasets_provider()
            return cls.datasets
        key = (model_cfg.seq_length, model_cfg.vocab_size, seed)
        if cls.datasets is None or cls._mock_key != key:
            cls.datasets = (MockGPTDataset(1 << 40, model_cfg.seq_length, model_cfg.vocab_size, seed), None, None)
            cls._mock_key = key
        return cls.datasets

    @classmethod
    def build_iterators(cls, training_state, consumed_samples: int):
        """Train iterator for this rank under the training state's strategy (valid/test: None)."""
        from ..models.llama import cp_positions

        ts = training_state
        ps = ts.ps
        train_ds = cls.get_datasets(ts.cfg, ts.train_cfg.seed)[0]
        s = ts.strategy
        pos = None
        if s.context_parallel_size > 1:
            pos = cp_positions(ts.cfg.seq_length, s.context_parallel_size, ps.cp_rank)
        from .hetero_dp import hetero_alignment

        sampler = PretrainingSampler(len(train_ds), consumed_samples, ts.train_cfg.micro_batch_size, ps.dp_rank,
                                     ps.dp_size, ts.train_cfg.global_batch_size, hetero_alignment())
        return DataIterator(train_ds, sampler, pos), None, None
