"""Tensor-parallel collectives fused with their GEMMs over NVLink peer memory.

``gemm_reduce_scatter`` replaces "GEMM, then NCCL reduce-scatter" (row-parallel forward and column-parallel
dgrad under sequence parallelism): one tcgen05 GEMM launch whose epilogue writes every finished output tile
straight into the owning TP rank's staging buffer (peer stores through CUDA-IPC mappings), so the NVLink
transfer overlaps the math of the remaining tiles; each rank then sums its TP slots with one small kernel.

Staging buffers are "symmetric": one ``cudaMalloc`` arena per rank of the TP group, mapped into every peer
once (``SymmetricBuffer``), grown on demand.  Ordering uses two stream-ordered 1-element NCCL all-reduces
per call (no device spin-waits): before the GEMM (every rank finished reading its staging from the previous
call) and after it (every partial tile has landed).

Disabled with ``EMB_FUSED_TP=0`` (then the plain GEMM + NCCL path runs).
"""
from __future__ import annotations

import os
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from .native import ext


class SymmetricBuffer:
    def __init__(self, group, nbytes: int, device: torch.device):
        self.group = group
        ranks = dist.get_process_group_ranks(group)
        self.n = len(ranks)
        self.idx = ranks.index(dist.get_rank())
        self.nbytes = nbytes
        self.arena = ext().arena_alloc(nbytes, device.index)
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
        self.peers = torch.tensor(ptrs, dtype=torch.int64)
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)

    def view(self, dtype, numel: int) -> torch.Tensor:
        return self.arena[: numel * torch.finfo(dtype).bits // 8].view(dtype)

    def close(self):
        for i, hh in enumerate(self.handles):
            if i != self.idx:
                ext().ipc_close(torch.frombuffer(bytearray(hh), dtype=torch.uint8))


_BUFS: Dict[Tuple[int, int], SymmetricBuffer] = {}


def _buffer(group, nbytes: int, device) -> SymmetricBuffer:
    key = (id(group), device.index)
    b = _BUFS.get(key)
    if b is None or b.nbytes < nbytes:
        if b is not None:
            # every rank of the group grows at the same call (same shapes), so the swap stays collective
            dist.all_reduce(b.flag, group=group)
            torch.cuda.synchronize(device)
            b.close()
        b = SymmetricBuffer(group, max(nbytes, 64 << 20), device)
        _BUFS[key] = b
    return b


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
    dist.all_reduce(buf.flag, group=group)  # peers finished reading their staging from the previous call
    ext().gemm_rs(a, b, trans_a, trans_b, buf.peers, buf.idx, rows)
    dist.all_reduce(buf.flag, group=group)  # every partial tile has landed in its owner's staging
    return ext().rs_reduce(buf.view(torch.bfloat16, tp * rows * N), tp, rows, N)


_READY: Dict[Tuple[int, int], torch.Tensor] = {}


def ag_eligible(shard: torch.Tensor, b: torch.Tensor, trans_b: bool, group) -> bool:
    if not (shard.is_cuda and enabled() and group is not None):
        return False
    tp = dist.get_world_size(group)
    return (1 < tp <= 8 and shard.dim() == 2 and shard.shape[0] % 256 == 0 and shard.shape[1] % 8 == 0
            and ext().gemm_tc_supported(shard, b, False, trans_b))


def all_gather_gemm(shard: torch.Tensor, b: torch.Tensor, trans_b: bool, group):
    """(all_gather(shard) @ op(b), gathered) over ``group``; ``gathered`` [tp * rows, K] stays valid until the
    next fused call on this group.

    The rank's own shard is placed in its symmetric buffer; one GEMM launch pulls the peers' shards over NVLink
    while it computes (copy warps inside the GEMM, chunk readiness counters, tiles of the local shard first).
    """
    tp = dist.get_world_size(group)
    R, K = shard.shape
    M = tp * R
    buf = _buffer(group, M * K * 2, shard.device)
    local = buf.view(torch.bfloat16, M * K).view(M, K)
    dist.all_reduce(buf.flag, group=group)  # peers finished with my buffer (previous fused call)
    local[buf.idx * R:(buf.idx + 1) * R].copy_(shard)
    dist.all_reduce(buf.flag, group=group)  # every rank's shard is in place
    key = (id(group), shard.device.index)
    ready = _READY.get(key)
    if ready is None:
        ready = torch.zeros(2 * tp, dtype=torch.int32, device=shard.device)
        _READY[key] = ready
    ready.zero_()
    y = ext().gemm_ag(local, b, trans_b, buf.peers, buf.idx, R, ready)
    return y, local
