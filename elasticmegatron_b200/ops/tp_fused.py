"""Tensor-parallel collectives fused with their GEMMs over NVLink peer memory.

``gemm_reduce_scatter`` replaces "GEMM, then NCCL reduce-scatter" (row-parallel forward and column-parallel
dgrad under sequence parallelism): one tcgen05 GEMM launch whose epilogue writes every finished output tile
straight into the owning TP rank's staging buffer (peer stores through CUDA-IPC mappings), so the NVLink
transfer overlaps the math of the remaining tiles; each rank then sums its TP slots with one small kernel.

Staging buffers are "symmetric": one ``cudaMalloc`` arena per rank of the TP group, mapped into every peer
once (``SymmetricBuffer``), grown on demand.  Each arena holds signal / flag arrays and two staging halves used
on alternate calls (call i uses half i % 2).

``all_gather_gemm`` pushes: the GEMM's copy warps store this rank's shard into every peer's half over NVLink
in 32-row units and release a per-unit flag (= the call's epoch) in the peer's flag array; a tile waits only
for the units of its own rows.  It needs no barrier.  ``gemm_reduce_scatter`` has one stream-ordered barrier
over the signal arrays after its GEMM (``sym_barrier``: peer stores of an epoch + bounded acquire spins; no
NCCL): every partial tile has landed before the local reduction.

Why two halves suffice without a "peers finished reading" barrier: a rank starts call i only after its call
i-1 finished, and call i-1 finished only after every peer took part in it (the reduce-scatter barrier, or the
peers' pushes that its all-gather GEMM waited for, which the peers issue from inside their own call-(i-1)
kernel).  So every peer has finished call i-2 - the last user of half i % 2 - before any rank writes that
half in call i.

Disabled with ``EMB_FUSED_TP=0`` (then the plain GEMM + NCCL path runs).
"""
from __future__ import annotations

import os
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from .native import ext


# Head of every arena: barrier signals (uint32 per rank) in the first 4 KiB, then the all-gather readiness flags
# (uint32 per (source chunk, unit of 32 rows)); the staging halves follow, 4 KiB aligned.
_SIG_BYTES = 64 << 10
_FLAG_OFF = 4096
_AG_UNIT_ROWS = 32
_AG_UNITS_MAX = (_SIG_BYTES - _FLAG_OFF) // 4 // 8
_TIMEOUT_MS = int(os.environ.get("EMB_FUSED_TP_TIMEOUT_MS", "60000"))


class SymmetricBuffer:
    def __init__(self, group, half_bytes: int, device: torch.device):
        self.group = group
        ranks = dist.get_process_group_ranks(group)
        self.ranks = tuple(ranks)
        self.n = len(ranks)
        self.idx = ranks.index(dist.get_rank())
        half_bytes = (half_bytes + 4095) // 4096 * 4096
        self.half = half_bytes
        self.nbytes = _SIG_BYTES + 2 * half_bytes
        self.arena = ext().arena_alloc(self.nbytes, device.index)
        self.arena[:_SIG_BYTES].zero_()
        torch.cuda.synchronize(device)  # signals are zero on every rank before any peer can map them
        h = bytes(ext().ipc_get_handle(self.arena).numpy().tobytes())
        handles = [None] * self.n
        dist.all_gather_object(handles, h, group=group)
        self.handles = handles
        ptrs = []
        for i, hh in enumerate(handles):
            if i == self.idx:
                ptrs.append(self.arena.data_ptr())
            else:
                ptrs.append(int(ext().ipc_open(torch.frombuffer(bytearray(hh), dtype=torch.uint8))))
        self.sig = torch.tensor(ptrs, dtype=torch.int64)
        self.flags = torch.tensor([p + _FLAG_OFF for p in ptrs], dtype=torch.int64)
        self.peers = [torch.tensor([p + _SIG_BYTES + h * half_bytes for p in ptrs], dtype=torch.int64)
                      for h in (0, 1)]
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)
        self.epoch = 0
        self.calls = 0
        self.closed = False

    def next_half(self) -> int:
        h = self.calls & 1
        self.calls += 1
        return h

    def barrier(self) -> None:
        self.epoch += 1
        ext().sym_barrier(self.sig, self.idx, self.epoch, _TIMEOUT_MS)

    def view(self, half: int, dtype, numel: int) -> torch.Tensor:
        off = _SIG_BYTES + half * self.half
        return self.arena[off: off + numel * torch.empty((), dtype=dtype).element_size()].view(dtype)

    def close(self):
        # holders of this object (e.g. a peer-memory DDP) see ``closed`` and rebuild on the new buffer
        self.closed = True
        for i, hh in enumerate(self.handles):
            if i != self.idx:
                ext().ipc_close(torch.frombuffer(bytearray(hh), dtype=torch.uint8))


_BUFS: Dict[Tuple[int, int], SymmetricBuffer] = {}


def _buffer(group, nbytes: int, device, tag: str = "", min_bytes: int = 64 << 20) -> SymmetricBuffer:
    """The group's symmetric buffer named ``tag``, grown (collectively) to at least ``nbytes`` per half.

    Growing replaces the buffer: the old one's peer mappings are closed, so callers look the buffer up at every
    use and never keep a ``SymmetricBuffer`` across calls that may grow it."""
    key = (id(group), device.index, tag)
    b = _BUFS.get(key)
    if b is None or b.half < nbytes:
        grow = 0
        if b is not None:
            # every rank of the group grows at the same call (same shapes), so the swap stays collective;
            # nobody may still read or write the old arenas when they are unmapped and freed
            dist.all_reduce(b.flag, group=group)
            torch.cuda.synchronize(device)
            b.close()
            grow = nbytes + nbytes // 4  # headroom: sizes that vary from call to call settle after a few grows
        b = SymmetricBuffer(group, max(nbytes, min_bytes, grow), device)
        _BUFS[key] = b
    return b


def release_buffers() -> None:
    """Unmap and free every symmetric buffer of this process (all ranks call it together, e.g. before the NCCL
    communicators are re-created).  Buffers are visited in one global order (by rank set, then name) and each
    is fenced by two barriers on its own group: nobody still uses a peer's arena when it is unmapped, and
    nobody frees its arena while a peer still maps it."""
    if not _BUFS:
        return
    for key, b in sorted(_BUFS.items(), key=lambda kv: (kv[1].ranks, kv[0][2])):
        torch.cuda.synchronize(b.arena.device)
        dist.all_reduce(b.flag, group=b.group)
        torch.cuda.synchronize(b.arena.device)
        b.close()
        dist.all_reduce(b.flag, group=b.group)
        torch.cuda.synchronize(b.arena.device)
    _BUFS.clear()
    _READY.clear()


def enabled() -> bool:
    return os.environ.get("EMB_FUSED_TP", "1") != "0"


def eligible(a: torch.Tensor, b: torch.Tensor, trans_a: bool, trans_b: bool, group) -> bool:
    if not (a.is_cuda and enabled() and group is not None):
        return False
    tp = dist.get_world_size(group)
    M = a.shape[1] if trans_a else a.shape[0]
    N = b.shape[0] if trans_b else b.shape[1]
    return tp > 1 and tp <= 8 and M % tp == 0 and N % 8 == 0 and ext().gemm_tc_supported(a, b, trans_a, trans_b)


def gemm_reduce_scatter(a: torch.Tensor, b: torch.Tensor, trans_a: bool, trans_b: bool, group) -> torch.Tensor:
    """reduce_scatter(op(a) @ op(b)) over ``group`` along rows; returns this rank's [M / tp, N] bf16 block."""
    tp = dist.get_world_size(group)
    M = a.shape[1] if trans_a else a.shape[0]
    N = b.shape[0] if trans_b else b.shape[1]
    rows = M // tp
    buf = _buffer(group, tp * rows * N * 2, a.device)
    h = buf.next_half()
    ext().gemm_rs(a, b, trans_a, trans_b, buf.peers[h], buf.idx, rows)
    buf.barrier()  # every partial tile has landed in its owner's staging
    return ext().rs_reduce(buf.view(h, torch.bfloat16, tp * rows * N), tp, rows, N)


_READY: Dict[Tuple[int, int], torch.Tensor] = {}


def ag_eligible(shard: torch.Tensor, b: torch.Tensor, trans_b: bool, group) -> bool:
    if not (shard.is_cuda and enabled() and group is not None):
        return False
    tp = dist.get_world_size(group)
    return (1 < tp <= 8 and shard.dim() == 2 and shard.shape[0] % 256 == 0 and shard.shape[1] % 8 == 0
            and shard.shape[0] // _AG_UNIT_ROWS <= _AG_UNITS_MAX and shard.is_contiguous()
            and ext().gemm_tc_supported(shard, b, False, trans_b))


def all_gather_gemm(shard: torch.Tensor, b: torch.Tensor, trans_b: bool, group):
    """(all_gather(shard) @ op(b), gathered) over ``group``; ``gathered`` [tp * rows, K] stays valid until the
    second-next fused call on this group (it lives in one staging half).

    The rank's own shard is placed in its own buffer; one GEMM launch pushes it into the peers' buffers over
    NVLink while it computes (copy warps inside the GEMM, per-unit readiness flags, tiles of the local shard
    first).
    """
    tp = dist.get_world_size(group)
    R, K = shard.shape
    M = tp * R
    buf = _buffer(group, M * K * 2, shard.device)
    h = buf.next_half()
    local = buf.view(h, torch.bfloat16, M * K).view(M, K)
    local[buf.idx * R:(buf.idx + 1) * R].copy_(shard)
    key = (id(group), shard.device.index)
    claim = _READY.get(key)
    if claim is None:
        claim = torch.zeros(1, dtype=torch.int32, device=shard.device)
        _READY[key] = claim
    claim.zero_()
    y = ext().gemm_ag(local, b, trans_b, buf.peers[h], buf.idx, R, claim, shard, buf.flags, buf.calls,
                      _AG_UNITS_MAX)
    return y, local
