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

Guard words (``EMB_ARENA_GUARD=1``): every arena gets ``GUARD_BYTES`` past its requested size filled with
``GUARD_FILL``; :func:`check_guards` (run by the manager after each switch and by ``train_step`` after each
step while enabled) raises if any live arena's tail changed, i.e. a transfer task or a kernel wrote past the
end of the state it was given.  This stands in for a sanitizer's out-of-bounds check on state arenas.
"""
from __future__ import annotations

import os
import weakref
from typing import Dict, List, Optional

import torch

GUARD_BYTES = 4096
GUARD_FILL = 0xA5


def guard_enabled() -> bool:
    return os.environ.get("EMB_ARENA_GUARD", "0") not in ("", "0")

_ELEM = {torch.float32: 4, torch.bfloat16: 2, torch.float16: 2, torch.uint8: 1, torch.int64: 8}


class Arena:
    """One flat allocation.  ``raw`` is a uint8 tensor over the whole allocation."""

    _next_id = 0

    def __init__(self, raw: torch.Tensor, nbytes: int, native: bool):
        self.raw, self.nbytes, self.native = raw, nbytes, native
        self.used = nbytes  # bytes requested by the current owner (views never extend past it)
        self.guard = 0  # guard bytes armed right after ``used``
        self.id = Arena._next_id
        Arena._next_id += 1
        self._ipc = None

    def view(self, dtype, shape) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        assert n * _ELEM[dtype] <= self.used, (shape, dtype, self.used)
        return self.raw[: n * _ELEM[dtype]].view(dtype).view(shape)

    def arm_guard(self, nbytes: int) -> None:
        self.guard = nbytes
        self.raw[self.used:self.used + nbytes].fill_(GUARD_FILL)

    def guard_intact(self) -> bool:
        if not self.guard:
            return True
        return bool((self.raw[self.used:self.used + self.guard] == GUARD_FILL).all().item())

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
        self.guard = GUARD_BYTES if guard_enabled() else 0
        self._live: "weakref.WeakSet[Arena]" = weakref.WeakSet()

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
        used = nbytes
        nbytes = self._round(used + self.guard)
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
        a.used = used
        if zero:
            a.raw.zero_()
        if self.guard:
            a.arm_guard(self.guard)
        self._live.add(a)
        return a

    def free(self, a: Optional[Arena]) -> None:
        if a is None:
            return
        self._live.discard(a)
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


def check_guards(where: str = "") -> None:
    """Raise if a guard word of any live arena of any pool was overwritten (no-op unless guards are armed)."""
    bad = []
    for key, pool in _POOLS.items():
        for a in list(pool._live):
            if not a.guard_intact():
                bad.append(f"arena {a.id} on {key} ({a.used} bytes used)")
    if bad:
        raise RuntimeError(f"state arena guard words overwritten{' after ' + where if where else ''}: " + "; ".join(bad))
