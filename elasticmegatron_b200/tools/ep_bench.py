"""MoE token movement under expert parallelism: peer-memory dispatch / combine against NCCL all-to-all.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m elasticmegatron_b200.tools.ep_bench --tokens 4096

One forward movement of an MoE layer = dispatch (every token's k rows to the ranks that own the chosen experts,
landing in the expert-grouped layout the grouped GEMM reads) + combine (expert outputs back to the token's
rank, weighted sum over the k choices).  The expert MLP itself is left out; the identity stands in for it.

* ``peer``: ``ops/ep_comm.py`` (counts all-gather read on the host, one push kernel, barrier, one return
  kernel, barrier, weighted gather);
* ``nccl``: the NCCL path of the MoE layer (counts all-to-all read on the host, local re-layout, all-to-all,
  local re-layout into the padded expert layout, and the same three steps back).

Timed with CUDA events on the compute stream after warm-up, MAX over ranks.  Roofline: max over GPUs of the
bytes that must cross NVLink (rows leaving or entering the GPU, both movements) / the link rate (nominal 900 GB/s per direction).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--link-gbs", type=float, default=900.0, help="link rate per direction (nominal NVLink 5: 900 GB/s; pass a measured rate to compare)")
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from ..models.moe import _layout, all_to_all
    from ..ops import ep_comm
    from ..ops.native import ext

    g = dist.group.WORLD
    ep, me = dist.get_world_size(), dist.get_rank()
    E, k, T, H = a.experts, a.topk, a.tokens, a.hidden
    e_loc = E // ep
    torch.manual_seed(1 + me)
    h = torch.randn(T, H, device="cuda").bfloat16()
    scores = torch.rand(T, E, device="cuda")
    top = scores.topk(k, -1).indices.to(torch.int32).contiguous()
    probs = torch.softmax(scores.gather(1, top.long()), -1)
    counts = torch.bincount(top.reshape(-1).long(), minlength=E).to(torch.int32)

    def peer():
        plan = ep_comm.EPPlan(g, top, counts, e_loc, H)
        xe = plan.push(h, None, with_origin=True)
        y = plan.send_home(xe)
        return ext().moe_gather(y, plan.ident, probs.reshape(-1).contiguous(), T, k)

    def nccl():
        gid = top.reshape(-1)
        send = _layout(gid, counts, T * k, 1)
        xs = ext().moe_scatter(h, k, send["pos"], None, send["seg"], send["counts"], send["cap"])
        cnt = counts.view(ep, e_loc)
        recv = torch.empty_like(cnt)
        dist.all_to_all_single(recv, cnt.contiguous(), group=g)
        ss, rs = cnt.sum(1).tolist(), recv.sum(1).tolist()
        xr = all_to_all(xs, ss, rs, g)
        n = int(sum(rs))
        gr = torch.repeat_interleave(torch.arange(e_loc, device="cuda", dtype=torch.int32).repeat(ep),
                                     recv.reshape(-1).to(torch.int64), output_size=n)
        lay = _layout(gr, recv.sum(0), n, 128)
        xe = ext().moe_scatter(xr, 1, lay["pos"], None, lay["seg"], lay["counts"], lay["cap"])
        yr = ext().moe_gather(xe, lay["pos"], None, n, 1)
        ys = all_to_all(yr, rs, ss, g)
        return ext().moe_gather(ys, send["pos"], probs.reshape(-1).float().contiguous(), T, k)

    torch.testing.assert_close(peer().float(), nccl().float(), atol=0, rtol=0)

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    t_p, t_n = timed(peer), timed(nccl)
    # rows that leave / enter each GPU in one dispatch (combine moves the same rows back)
    allc = torch.empty(ep, E, dtype=torch.int32, device="cuda")
    dist.all_gather_into_tensor(allc, counts, group=g)
    ac = allc.cpu().long()
    eg = ac.view(ep, ep, e_loc).sum(2)  # [src, dst] rows
    out_rows = (eg.sum(1) - eg.diagonal()).max().item()
    in_rows = (eg.sum(0) - eg.diagonal()).max().item()
    roof = 2 * max(out_rows, in_rows) * H * 2 / (a.link_gbs * 1e9) * 1e3
    if me == 0:
        print(json.dumps({"ep": ep, "tokens": T, "hidden": H, "experts": E, "topk": k, "peer_ms": t_p,
                          "nccl_ms": t_n, "speedup": t_n / t_p, "roofline_ms": roof, "peer_roofline_frac": roof / t_p,
                          "error_flag": int(ext().comm_error_flag())}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
