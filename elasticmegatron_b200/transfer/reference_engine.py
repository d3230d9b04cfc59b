"""The reference's transfer *algorithm*, re-implemented on this framework's layouts (NCCL / Gloo baseline).

This is not the reference's own build (that needs Megatron-LM); it reproduces its communication schedule
so a same-box baseline exists for the reshard latency metric (elastic_megatron/transfer/transfer.py:143-341):

1. **pre** - for every virtual parameter, every ZeRO shard of each source TP shard is sent to the *aligned*
   source rank (the lowest shard index holding part of it), which assembles the padded full TP-local fp32
   master / exp_avg / exp_avg_sq;
2. **main** - each aligned source rank sends every destination TP chunk that overlaps its TP shard to the
   aligned destination rank, which assembles the full destination TP-local tensors; TP-replicated
   parameters go from the TP-rank-0 copy to every destination TP rank (resharding_tp.py:119-139);
3. **post** - the aligned destination rank scatters each destination ZeRO shard to its owner;

every (parameter, tensor, peer) exchange is its own blocking point-to-point call, in a fixed global order.
Afterwards the bf16 parameters are regenerated from the master of the own shard and all-gathered over DP
(``TrainingState.update_model_weight``, training_state.py:176-197); the manager does that because this
engine sets ``moves_params = False``.
"""
from __future__ import annotations

from typing import Dict, List

import torch
import torch.distributed as dist

from ..config import get_args
from ..planner.layout import virtual_params
from ..planner.plan import ReshardPlan, _StrategyView, _intersect


def _numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


class ReferenceAlgorithmEngine:
    name = "reference_algorithm"
    moves_params = False

    def __init__(self, send_fn=None, recv_fn=None, broadcast_fn=None, use_p2p_to_collective: bool = False):
        """``send_fn(t, dst)`` / ``recv_fn(t, src)`` / ``broadcast_fn(t, src, group)`` replace the NCCL calls
        (the reference's injectable communicator, elastic_manager.py:41-51); with ``use_p2p_to_collective`` a
        point-to-point exchange is a broadcast on the 2-rank group {src, dst} (p2p_to_collective.py:41-96)."""
        self.bytes_sent = 0
        self.send_fn = send_fn or (lambda t, dst: dist.send(t, dst))
        self.recv_fn = recv_fn or (lambda t, src: dist.recv(t, src))
        self.broadcast_fn = broadcast_fn or (lambda t, src, group: dist.broadcast(t, src=src, group=group))
        self.use_p2p_to_collective = use_p2p_to_collective

    def reset_counters(self):
        self.bytes_sent = 0

    def execute(self, plan: ReshardPlan, rank: int, sp, so, dp, do, group=None) -> None:
        args = get_args()
        cfg, tc = args.model, args.train
        sv = _StrategyView(cfg, plan.src, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        dv = _StrategyView(cfg, plan.dst, tc.overlap_grad_reduce, tc.ddp_bucket_size)
        dev = (so if so is not None else do).device
        for vp in virtual_params(cfg):
            src_groups = self._tp_groups(sv, vp, sv.holders(vp), True)
            dst_groups = self._tp_groups(dv, vp, dv.holders(vp), False)
            full_src: Dict[int, torch.Tensor] = {}
            # pre: gather ZeRO shards onto the aligned source rank of each TP shard
            for key, ranks in sorted(src_groups.items()):
                aligned = ranks[0]
                shape = sv.layouts[aligned].vp_loc[vp.index][1]
                if rank == aligned:
                    full_src[key] = torch.zeros((3, _numel(shape)), dtype=torch.float32, device=dev)
                for r in ranks:
                    self._gather_piece(sv, vp, r, aligned, rank, so, full_src.get(key), dev)
            # main: aligned src -> aligned dst per overlapping TP chunk
            full_dst: Dict[int, torch.Tensor] = {}
            for dkey, dranks in sorted(dst_groups.items()):
                dal = dranks[0]
                dshape = dv.layouts[dal].vp_loc[vp.index][1]
                if rank == dal:
                    full_dst[dkey] = torch.zeros((3, _numel(dshape)), dtype=torch.float32, device=dev)
                dpieces = dv.param_pieces(vp, dal)
                for skey, sranks in sorted(src_groups.items()):
                    sal = sranks[0]
                    self._move_boxes(sal, dal, sv.param_pieces(vp, sal), dpieces, rank, full_src.get(skey),
                                     full_dst.get(dkey), sv.layouts[sal].vp_loc[vp.index][0],
                                     dv.layouts[dal].vp_loc[vp.index][0], dev)
            # post: scatter from the aligned destination rank to every ZeRO owner
            for dkey, dranks in sorted(dst_groups.items()):
                for r in dranks:
                    self._scatter_piece(dv, vp, r, dranks[0], rank, do, full_dst.get(dkey), dev)
        if dev.type == "cuda":
            torch.cuda.synchronize()

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _tp_groups(view, vp, holders, is_src: bool) -> Dict[tuple, List[int]]:
        """Ranks holding each TP shard (instance 0 only), ordered by ZeRO shard index, keyed (stage, TP rank).

        A tied embedding has a copy on the first and on the last stage: the source side reads the first
        stage's, the destination side fills both (the reference re-broadcasts the word embedding to the last
        stage over the embedding group, transfer/transfer.py:103-141)."""
        if is_src and holders:
            first = min(view.coords[r]["pp"] for r in holders)
            holders = [r for r in holders if view.coords[r]["pp"] == first]
        out: Dict[tuple, List[int]] = {}
        for r in holders:
            if view.layouts[r].instance != 0:
                continue
            c = view.coords[r]
            out.setdefault((c["pp"], c["etp"] if vp.is_expert else c["tp"]), []).append(r)
        for t in out:
            out[t].sort(key=lambda r: (view.layouts[r].expert_shard_index if vp.is_expert
                                       else view.layouts[r].dense_shard_index, r))
        if vp.tp_dim is None and is_src:
            out = {k: v for k, v in out.items() if k[1] == 0}
        return out

    @staticmethod
    def _owned_ranges(view, vp, r):
        rl = view.layouts[r]
        P, shape = rl.vp_loc[vp.index]
        n = _numel(shape)
        out = []
        for s, e, o in rl.owned():
            lo, hi = max(s, P), min(e, P + n)
            if lo < hi:
                out.append((lo - P, hi - P, o + (lo - s)))
        return out

    def _p2p(self, t: torch.Tensor, src: int, dst: int, rank: int):
        if src == dst or rank not in (src, dst):
            return
        if self.use_p2p_to_collective:
            from ..parallel.process_groups import ProcessGroupPool

            buf = t.contiguous()
            pair = ProcessGroupPool.get(sorted((src, dst)))
            if pair is None:
                raise RuntimeError(f"no process group for ranks {{{src}, {dst}}}: construct the manager with "
                                   "use_p2p_to_collective=True on every rank so the pair groups exist")
            self.broadcast_fn(buf, src, pair)
            if rank == dst and buf.data_ptr() != t.data_ptr():
                t.copy_(buf)
            if rank == src:
                self.bytes_sent += t.numel() * t.element_size()
            return
        if rank == src:
            self.send_fn(t.contiguous(), dst)
            self.bytes_sent += t.numel() * t.element_size()
        else:
            buf = t if t.is_contiguous() else torch.empty_like(t, memory_format=torch.contiguous_format)
            self.recv_fn(buf, src)
            if buf is not t:
                t.copy_(buf)

    def _gather_piece(self, view, vp, r, aligned, rank, opt, full, dev):
        for f0, f1, o in self._owned_ranges(view, vp, r):
            n = f1 - f0
            for k in range(3):
                if r == aligned:
                    if rank == r:
                        full[k, f0:f1].copy_(opt[k, o:o + n])
                    continue
                if rank == r:
                    self._p2p(opt[k, o:o + n], r, aligned, rank)
                elif rank == aligned:
                    buf = torch.empty(n, dtype=torch.float32, device=dev)
                    self._p2p(buf, r, aligned, rank)
                    full[k, f0:f1].copy_(buf)

    def _scatter_piece(self, view, vp, r, aligned, rank, opt, full, dev):
        for f0, f1, o in self._owned_ranges(view, vp, r):
            n = f1 - f0
            for k in range(3):
                if r == aligned:
                    if rank == r:
                        opt[k, o:o + n].copy_(full[k, f0:f1])
                    continue
                if rank == aligned:
                    self._p2p(full[k, f0:f1].contiguous(), aligned, r, rank)
                elif rank == r:
                    buf = torch.empty(n, dtype=torch.float32, device=dev)
                    self._p2p(buf, aligned, r, rank)
                    opt[k, o:o + n].copy_(buf)

    def _move_boxes(self, sal, dal, spieces, dpieces, rank, sfull, dfull, sbase, dbase, dev):
        for spc in spieces:
            for dpc in dpieces:
                box = _intersect(spc, dpc)
                if box is None:
                    continue
                r0, r1, c0, c1 = box
                rows, cols = r1 - r0, c1 - c0
                so = spc.off(r0, c0) - sbase
                do = dpc.off(r0, c0) - dbase
                for k in range(3):
                    src = dst = None
                    if rank == sal:
                        src = sfull[k].as_strided((rows, cols), (spc.ld, 1), sfull[k].storage_offset() + so)
                    if rank == dal:
                        dst = dfull[k].as_strided((rows, cols), (dpc.ld, 1), dfull[k].storage_offset() + do)
                    if sal == dal:
                        if rank == sal:
                            dst.copy_(src)
                        continue
                    if rank == sal:
                        self._p2p(src.contiguous(), sal, dal, rank)
                    elif rank == dal:
                        buf = torch.empty((rows, cols), dtype=torch.float32, device=dev)
                        self._p2p(buf, sal, dal, rank)
                        dst.copy_(buf)
