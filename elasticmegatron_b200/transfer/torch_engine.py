"""Transfer engine over ``torch.distributed`` point-to-point (NCCL on GPU, Gloo on CPU).

Executes a :class:`~elasticmegatron_b200.planner.plan.ReshardPlan` with one packed message per
(peer, kind): descriptors bound for the same peer are packed into one contiguous buffer, and all sends and
receives of the switch are posted at once with ``batch_isend_irecv``.  This is the CPU path and the
NCCL-only baseline; the reference instead issues one blocking 2-rank NCCL broadcast per (param, tensor,
peer) in three phases (elastic_megatron/transfer/transfer.py:291-341, p2p_to_collective.py:44-96), which
``transfer/reference_engine.py`` reproduces for comparison.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from ..planner.plan import KIND_OPT, KIND_PARAM, ReshardPlan


def _view(flat: torch.Tensor, off: int, rows: int, cols: int, stride: int) -> torch.Tensor:
    if rows == 1:
        return flat[off:off + cols]
    return flat.as_strided((rows, cols), (stride, 1), flat.storage_offset() + off)


def _opt_view(opt: torch.Tensor, off: int, rows: int, cols: int, stride: int) -> torch.Tensor:
    # opt: [3, n]
    if rows == 1:
        return opt[:, off:off + cols]
    n = opt.stride(0)
    return opt.as_strided((3, rows, cols), (n, stride, 1), opt.storage_offset() + off)


class TorchP2PEngine:
    name = "torch_p2p"

    def __init__(self):
        self.bytes_sent = 0
        self.bytes_recv = 0

    def reset_counters(self):
        self.bytes_sent = self.bytes_recv = 0

    def execute(self, plan: ReshardPlan, rank: int, src_param: Optional[torch.Tensor],
                src_opt: Optional[torch.Tensor], dst_param: Optional[torch.Tensor],
                dst_opt: Optional[torch.Tensor], group=None) -> None:
        d = plan.desc
        mine_s = d[(d["src_rank"] == rank)]
        mine_d = d[(d["dst_rank"] == rank)]
        # local copies
        loc = mine_s[mine_s["dst_rank"] == rank]
        for r in loc:
            self._copy_local(r, src_param, src_opt, dst_param, dst_opt)
        ops = []
        sends: List[Tuple[int, torch.Tensor]] = []
        recvs: List[Tuple[int, int, torch.Tensor, np.ndarray]] = []
        # sends grouped by (dst, kind)
        for (peer, kind), rows in _group(mine_s[mine_s["dst_rank"] != rank]).items():
            buf = self._pack(rows, kind, src_param, src_opt)
            sends.append((peer, buf))
            ops.append(dist.P2POp(dist.isend, buf, peer, group))
            self.bytes_sent += buf.numel() * buf.element_size()
        for (peer, kind), rows in _group(mine_d[mine_d["src_rank"] != rank], key="src_rank").items():
            n = int((rows["rows"] * rows["cols"]).sum())
            if kind == KIND_OPT:
                buf = torch.empty((3, n), dtype=dst_opt.dtype, device=dst_opt.device)
            else:
                buf = torch.empty((n,), dtype=dst_param.dtype, device=dst_param.device)
            recvs.append((peer, kind, buf, rows))
            ops.append(dist.P2POp(dist.irecv, buf, peer, group))
            self.bytes_recv += buf.numel() * buf.element_size()
        # deterministic op order: sort by (peer, send/recv) so both sides agree for gloo pairing
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        for peer, kind, buf, rows in recvs:
            self._unpack(rows, kind, buf, dst_param, dst_opt)

    # ------------------------------------------------------------------
    @staticmethod
    def _copy_local(r, sp, so, dp, do):
        rows, cols = int(r["rows"]), int(r["cols"])
        if r["kind"] == KIND_OPT:
            _opt_view(do, int(r["dst_off"]), rows, cols, int(r["dst_stride"])).copy_(
                _opt_view(so, int(r["src_off"]), rows, cols, int(r["src_stride"])))
        else:
            _view(dp, int(r["dst_off"]), rows, cols, int(r["dst_stride"])).copy_(
                _view(sp, int(r["src_off"]), rows, cols, int(r["src_stride"])))

    @staticmethod
    def _pack(rows, kind, sp, so) -> torch.Tensor:
        n = int((rows["rows"] * rows["cols"]).sum())
        if kind == KIND_OPT:
            buf = torch.empty((3, n), dtype=so.dtype, device=so.device)
            o = 0
            for r in rows:
                k = int(r["rows"] * r["cols"])
                buf[:, o:o + k].view(3, int(r["rows"]), int(r["cols"])).copy_(
                    _opt_view(so, int(r["src_off"]), int(r["rows"]), int(r["cols"]), int(r["src_stride"]))
                    .reshape(3, int(r["rows"]), int(r["cols"])))
                o += k
        else:
            buf = torch.empty((n,), dtype=sp.dtype, device=sp.device)
            o = 0
            for r in rows:
                k = int(r["rows"] * r["cols"])
                buf[o:o + k].view(int(r["rows"]), int(r["cols"])).copy_(
                    _view(sp, int(r["src_off"]), int(r["rows"]), int(r["cols"]), int(r["src_stride"]))
                    .reshape(int(r["rows"]), int(r["cols"])))
                o += k
        return buf

    @staticmethod
    def _unpack(rows, kind, buf, dp, do):
        o = 0
        for r in rows:
            k = int(r["rows"] * r["cols"])
            R, C = int(r["rows"]), int(r["cols"])
            if kind == KIND_OPT:
                _opt_view(do, int(r["dst_off"]), R, C, int(r["dst_stride"])).copy_(
                    buf[:, o:o + k].view(3, R, C) if R > 1 else buf[:, o:o + k])
            else:
                _view(dp, int(r["dst_off"]), R, C, int(r["dst_stride"])).copy_(
                    buf[o:o + k].view(R, C) if R > 1 else buf[o:o + k])
            o += k


def _group(rows: np.ndarray, key: str = "dst_rank") -> Dict[Tuple[int, int], np.ndarray]:
    out = {}
    if len(rows) == 0:
        return out
    order = np.lexsort((rows["vp"], rows["kind"], rows[key]))
    rows = rows[order]
    for peer in np.unique(rows[key]):
        for kind in (KIND_OPT, KIND_PARAM):
            sel = rows[(rows[key] == peer) & (rows["kind"] == kind)]
            if len(sel):
                out[(int(peer), kind)] = sel
    return out
