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
    """Size-keyed cache of released arenas.

    ``alloc`` reuses the smallest free arena that is at least the requested size and at most ``slack`` times
    larger (best fit), so alternating between layouts whose arenas differ only by padding reuses memory and
    peer mappings.  The free cache is bounded by ``max_cached_bytes`` (default: 40% of the device); older
    entries beyond it are returned to the driver, and a failed allocation trims the whole cache and retries.
    """

    def __init__(self, device: torch.device, max_cached_bytes: Optional[int] = None, slack: float = 1.25):
        self.device = torch.device(device)
        self._free: List[Arena] = []
        self.allocated_bytes = 0
        self.slack = slack
        if max_cached_bytes is None:
            total = 0
            if self.device.type == "cuda":
                total = torch.cuda.get_device_properties(self.device).total_memory
            max_cached_bytes = int(0.4 * total) if total else (1 << 62)
        self.max_cached_bytes = max_cached_bytes

    @staticmethod
    def _round(nbytes: int) -> int:
        g = 2 << 20
        return max(g, (nbytes + g - 1) // g * g)

    def cached_bytes(self) -> int:
        return sum(a.nbytes for a in self._free)

    def _new(self, nbytes: int) -> Arena:
        if self.device.type == "cuda":
            from ..ops.native import ext

            dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
            raw = ext().arena_alloc(nbytes, dev)
            return Arena(raw, nbytes, True)
        return Arena(torch.empty(nbytes, dtype=torch.uint8, device=self.device), nbytes, False)

    def alloc(self, nbytes: int, zero: bool = False) -> Arena:
        nbytes = self._round(nbytes)
        fits = [a for a in self._free if nbytes <= a.nbytes <= self.slack * nbytes]
        if fits:
            a = min(fits, key=lambda x: x.nbytes)
            self._free.remove(a)
        else:
            try:
                a = self._new(nbytes)
            except RuntimeError:
                self.trim()
                a = self._new(nbytes)
            self.allocated_bytes += nbytes
        if zero:
            a.raw.zero_()
        return a

    def free(self, a: Optional[Arena]) -> None:
        if a is None:
            return
        self._free.append(a)
        while self.cached_bytes() > self.max_cached_bytes and self._free:
            old = self._free.pop(0)
            self.allocated_bytes -= old.nbytes
            del old

    def trim(self) -> None:
        """Return every cached free arena to the driver."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for a in self._free:
            self.allocated_bytes -= a.nbytes
        self._free.clear()


_POOLS: Dict[str, ArenaPool] = {}


def get_pool(device) -> ArenaPool:
    key = str(torch.device(device))
    if key not in _POOLS:
        _POOLS[key] = ArenaPool(torch.device(device))
    return _POOLS[key]
