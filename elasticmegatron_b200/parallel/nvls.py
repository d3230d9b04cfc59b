"""All-reduce of fp32 tensors through NVSwitch multicast (NVLS ``multimem``), with a peer-memory fallback.

Used for the Group-ZeRO reduction of each gradient shard across optimizer instances (``ddp.py``; Megatron does it
with an NCCL all-reduce over the inter-instance group).  Every rank of the group holds one symmetric staging
buffer, allocated and mapped by PyTorch's symmetric-memory allocator (``torch.distributed._symmetric_memory``:
one physical allocation per GPU, peer mappings and, where the GPUs sit behind an NVSwitch with multicast, one
NVLink multicast object bound to all of them).  A tensor is reduced chunk by chunk:

    copy into the staging buffer -> barrier -> reduce my slice -> barrier -> copy out

``reduce my slice`` is ``nvls_allreduce_f32`` (``csrc/comm/nvls.cu``): ``multimem.ld_reduce`` returns the sum of
the slice over all GPUs, computed in the switch, and ``multimem.st`` writes it to every GPU's buffer.  Without a
multicast object it is ``p2p_allreduce_f32``: unicast peer loads in a fixed rank order and peer stores of the sum.
The barriers are ``sym_barrier`` (bounded peer-flag waits) over a signal area at the head of the same buffer.

Which one runs: per GPU, the multicast all-reduce moves about (n + 1) / n of the buffer in each direction (its
share of every slice to the switch, the reduced slice back, the broadcast results in), a ring 2 (n - 1) / n and the
peer-memory kernel (n - 1) / n plus its peer stores.  Multicast therefore pays from four GPUs up; at two it moves
1.5x the ring's bytes (measured on 2 B200s, 256 MB: NCCL 0.52 ms, peer memory 0.60 ms, multicast 0.86 ms, each
including the two local staging copies).  ``EMB_NVLS`` = ``1`` (default: multicast for groups of >= 4 GPUs where
the buffer has a multicast object, peer memory otherwise), ``nvls`` (multicast whenever available), ``p2p``, or
``0`` (NCCL all-reduce).  A test that makes a rank leave a GPU job must run with ``EMB_NVLS=0``: a process that dies
while its memory is bound to a multicast object can raise NVLink errors on the other GPUs of the object.
"""
from __future__ import annotations

import os
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from ..ops.native import ext

_SIG = 64 << 10  # signal head (one uint32 slot per rank for sym_barrier); keeps the data 64 KiB aligned
_CHUNK = int(os.environ.get("EMB_NVLS_CHUNK_MB", "64")) << 20
_TIMEOUT_MS = int(os.environ.get("EMB_NVLS_TIMEOUT_MS", "60000"))


def mode() -> str:
    """'auto', 'nvls' (multicast when the buffer has it, else peer memory), 'p2p' (peer memory) or 'off' (NCCL)."""
    v = os.environ.get("EMB_NVLS", "1").lower()
    if v in ("0", "off", "nccl"):
        return "off"
    return v if v in ("p2p", "nvls") else "auto"


class SymmetricAllReduce:
    """One group's staging buffer and the chunked all-reduce over it."""

    def __init__(self, group, device: torch.device, chunk_bytes: int = _CHUNK, force_p2p: bool = False):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        assert 1 <= self.n <= 8, "one NVSwitch domain (<= 8 GPUs)"
        self.chunk = (chunk_bytes + 4095) // 4096 * 4096
        self.buf = symm_mem.empty(_SIG + self.chunk, dtype=torch.uint8, device=device)
        self.buf[:_SIG].zero_()
        torch.cuda.synchronize(device)  # zero signals before any peer can reach them through the rendezvous
        self.handle = symm_mem.rendezvous(self.buf, group)
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        # the tensor may start inside the symmetric allocation; every rank's sits at the same offset
        off = self.buf.data_ptr() - ptrs[self.me]
        offs = [None] * self.n
        dist.all_gather_object(offs, off, group=group)
        assert all(o == off for o in offs), f"symmetric buffers at different offsets: {offs}"
        self.ptrs = torch.tensor([p + off for p in ptrs], dtype=torch.int64)
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self.mc = 0 if (force_p2p or not mc) else mc + off
        self.epoch = 0

    @property
    def kind(self) -> str:
        return "nvls" if self.mc else "p2p"

    def _barrier(self) -> None:
        self.epoch += 1
        ext().sym_barrier(self.ptrs, self.me, self.epoch, _TIMEOUT_MS)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """Sum ``t`` (fp32, contiguous, on this rank's GPU) over the group in place; stream-ordered on the current
        stream.  Every rank calls it with the same numel."""
        assert t.dtype == torch.float32 and t.is_contiguous() and t.is_cuda
        flat = t.view(-1)
        cap = self.chunk // 4
        for s in range(0, flat.numel(), cap):
            part = flat[s:s + cap]
            m = part.numel()
            stage = self.buf[_SIG:_SIG + 4 * m].view(torch.float32)
            stage.copy_(part)
            self._barrier()
            per = ((m + self.n - 1) // self.n + 3) // 4 * 4  # slices of whole 16-byte vectors
            lo = min(self.me * per, m)
            hi = min(lo + per, m)
            if hi > lo:
                if self.mc:
                    ext().nvls_allreduce_f32(self.mc + _SIG + 4 * lo, hi - lo)
                else:
                    ext().p2p_allreduce_f32(self.ptrs, _SIG + 4 * lo, hi - lo)
            self._barrier()
            part.copy_(stage)
        return t


_CACHE: Dict[Tuple[int, int, str], SymmetricAllReduce] = {}


def get(group, device: torch.device, kind: str = None) -> SymmetricAllReduce:
    """The cached reducer of ``group`` (built collectively on first use)."""
    kind = kind or mode()
    if kind == "auto":
        kind = "nvls" if dist.get_world_size(group) >= 4 else "p2p"
    key = (id(group), device.index, kind)
    r = _CACHE.get(key)
    if r is None:
        r = SymmetricAllReduce(group, device, force_p2p=kind == "p2p")
        _CACHE[key] = r
    return r


def all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    """In-place sum over ``group``: NVLS / peer memory for fp32 CUDA tensors of groups within one NVSwitch
    domain, NCCL otherwise (or with ``EMB_NVLS=0``)."""
    n = dist.get_world_size(group)
    if n == 1:
        return t
    if (mode() == "off" or not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous() or n > 8
            or dist.get_backend(group) != "nccl"):
        dist.all_reduce(t, group=group)
        return t
    return get(group, t.device).all_reduce_(t)


def release() -> None:
    """Drop every reducer (all ranks call it together, e.g. before process groups are re-created): in one global
    order, each group's ranks finish their work on the buffer and meet before it is freed."""
    for key, r in sorted(_CACHE.items(), key=lambda kv: (tuple(dist.get_process_group_ranks(kv[1].group)), kv[0][2])):
        torch.cuda.synchronize(r.buf.device)
        r._barrier()
        torch.cuda.synchronize(r.buf.device)
    _CACHE.clear()
