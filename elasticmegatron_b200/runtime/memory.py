"""Flat state arenas with a size-keyed free list.

Each strategy's state lives in three flat arenas per rank: parameters, fp32 gradients and the fp32
``[3, n]`` optimizer state.  Releasing a strategy returns its arenas to the pool and rebuilding takes
arenas back (views are re-pointed), which replaces the reference's ``untyped_storage().resize_(0)`` trick and
its per-switch ``torch.cuda.empty_cache()`` (elastic_megatron/megatron_manager/training_state.py:199-311;
elastic_manager.py:252, "50~100+ ms").

On CUDA the arenas are ``cudaMalloc`` allocations made by the native extension (not the caching allocator)
so each can be exported as one CUDA IPC handle and mapped by peer processes for the direct-transfer engine;
peer mappings are cached by the engine, and because the pool reuses arenas across switches the mappings
stay valid.
"""
from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Optional

import torch

_ELEM = {torch.float32: 4, torch.bfloat16: 2, torch.float16: 2, torch.uint8: 1, torch.int64: 8}


class Arena:
    """One flat allocation.  ``raw`` is a uint8 tensor over the whole allocation."""

    _next_id = 0

    def __init__(self, raw: torch.Tensor, nbytes: int, native: bool):
        self.raw, self.nbytes, self.native = raw, nbytes, native
        self.id = Arena._next_id
        Arena._next_id += 1
        self._ipc = None

    def view(self, dtype, shape) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        assert n * _ELEM[dtype] <= self.nbytes, (shape, dtype, self.nbytes)
        return self.raw[: n * _ELEM[dtype]].view(dtype).view(shape)

    @property
    def ptr(self) -> int:
        return self.raw.data_ptr()

    def ipc_handle(self) -> bytes:
        """CUDA IPC handle of the allocation (64 bytes)."""
        if self._ipc is None:
            from ..ops.native import ext

            self._ipc = bytes(ext().ipc_get_handle(self.raw))
        return self._ipc


class ArenaPool:
    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self._free: Dict[int, List[Arena]] = defaultdict(list)
        self.allocated_bytes = 0

    @staticmethod
    def _round(nbytes: int) -> int:
        g = 2 << 20
        return max(g, (nbytes + g - 1) // g * g)

    def alloc(self, nbytes: int, zero: bool = False) -> Arena:
        nbytes = self._round(nbytes)
        lst = self._free.get(nbytes)
        if lst:
            a = lst.pop()
        else:
            if self.device.type == "cuda":
                from ..ops.native import ext

                raw = ext().arena_alloc(nbytes, self.device.index if self.device.index is not None
                                        else torch.cuda.current_device())
                a = Arena(raw, nbytes, True)
            else:
                a = Arena(torch.empty(nbytes, dtype=torch.uint8, device=self.device), nbytes, False)
            self.allocated_bytes += nbytes
        if zero:
            a.raw.zero_()
        return a

    def free(self, a: Optional[Arena]) -> None:
        if a is not None:
            self._free[a.nbytes].append(a)

    def trim(self) -> None:
        """Drop cached free arenas (returns device memory)."""
        for lst in self._free.values():
            for a in lst:
                self.allocated_bytes -= a.nbytes
        self._free.clear()


_POOLS: Dict[str, ArenaPool] = {}


def get_pool(device) -> ArenaPool:
    key = str(torch.device(device))
    if key not in _POOLS:
        _POOLS[key] = ArenaPool(torch.device(device))
    return _POOLS[key]
