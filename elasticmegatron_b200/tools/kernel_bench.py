"""Kernel micro-benchmarks with CUDA-event timing and roofline fractions.

    python -m elasticmegatron_b200.tools.kernel_bench gemm --m 16384 --n 4096 --k 4096 --layout fprop
    python -m elasticmegatron_b200.tools.kernel_bench all
    python -m elasticmegatron_b200.tools.kernel_bench fused --m 4096 --n 4096 --k 4096

``fused`` runs the fused tensor-parallel kernels on ONE GPU with a 2-rank group emulated in local memory
(the "peer" staging / gather buffers are ordinary local allocations and the all-gather readiness flags of the
other rank's chunk are set before the launch), so the kernels can be profiled with single-GPU tools; the
NVLink side of the real kernels is measured by ``tp_bench``.

Each case runs a warm-up, then ``--iters`` timed launches bracketed by ``cuda.synchronize``, on inputs larger
than L2 where the op is memory-bound.  Fractions are reported against the measured peaks in
MEASURED_PEAKS.json at the repository root when present (``bf16_tflops``, ``hbm_gbs``), else the pool
fallback (1590 TFLOP/s, 6650 GB/s).  ``--baseline`` also times the torch / cuBLAS equivalent.
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def timeit(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def bench_gemm(m, n, k, layout, iters, baseline, variant=0):
    from elasticmegatron_b200.ops.native import ext

    dev = "cuda"
    if layout == "fprop":
        a, b = torch.randn(m, k, device=dev).bfloat16(), torch.randn(n, k, device=dev).bfloat16()
        fn = lambda: ext().gemm_tc(a, b, False, True, variant=variant)
        ref = lambda: torch.matmul(a, b.t())
    elif layout == "dgrad":
        a, b = torch.randn(m, k, device=dev).bfloat16(), torch.randn(k, n, device=dev).bfloat16()
        fn = lambda: ext().gemm_tc(a, b, False, False, variant=variant)
        ref = lambda: torch.matmul(a, b)
    elif layout == "tn":  # A MN-major, B K-major: a [K, M], b [N, K]
        a, b = torch.randn(k, m, device=dev).bfloat16(), torch.randn(n, k, device=dev).bfloat16()
        fn = lambda: ext().gemm_tc(a, b, True, True, variant=variant)
        ref = lambda: torch.matmul(a.t(), b.t())
    elif layout == "wgrad_bf16":  # both MN-major, bf16 output (no accumulate)
        a, b = torch.randn(k, m, device=dev).bfloat16(), torch.randn(k, n, device=dev).bfloat16()
        fn = lambda: ext().gemm_tc(a, b, True, False, variant=variant)
        ref = lambda: torch.matmul(a.t(), b)
    else:
        a, b = torch.randn(k, m, device=dev).bfloat16(), torch.randn(k, n, device=dev).bfloat16()
        c = torch.zeros(m, n, device=dev)
        fn = lambda: ext().gemm_tc(a, b, True, False, c, True, variant=variant)
        # the same work in cuBLAS: bf16 operands, fp32 C read and accumulated (beta = 1) into an fp32 output
        ref = lambda: torch.addmm(c, a.t(), b, out_dtype=torch.float32)
    ms = timeit(fn, iters)
    tf = 2 * m * n * k / ms / 1e9
    pk, _, src = peaks()
    out = {"op": f"gemm_{layout}", "variant": variant, "m": m, "n": n, "k": k, "ms": ms, "tflops": tf, "frac": tf / pk, "peak": src}
    if baseline:
        bms = timeit(ref, iters)
        out.update({"cublas_ms": bms, "cublas_tflops": 2 * m * n * k / bms / 1e9})
    return out


def bench_mem(name, fn, nbytes, iters):
    ms = timeit(fn, iters)
    _, hbm, src = peaks()
    gbs = nbytes / ms / 1e6
    return {"op": name, "ms": ms, "gbs": gbs, "frac": gbs / hbm, "peak": src}


def bench_elementwise(iters):
    from elasticmegatron_b200.ops.native import ext

    T, H, F = 32768, 4096, 11008
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    out = [bench_mem("rmsnorm_fwd", lambda: ext().rmsnorm_fwd(x, w, 1e-5), 2 * T * H * 2, iters)]
    y, rstd = ext().rmsnorm_fwd(x, w, 1e-5)
    out.append(bench_mem("rmsnorm_bwd", lambda: ext().rmsnorm_bwd(x, x, w, rstd), 3 * T * H * 2, iters))
    h = torch.randn(8192, 2 * F, device="cuda").bfloat16()
    out.append(bench_mem("swiglu_fwd", lambda: ext().swiglu_fwd(h), 8192 * 3 * F * 2, iters))
    n = 1 << 28
    O = torch.zeros(3, n, device="cuda")
    G = torch.zeros(n, device="cuda")
    P = torch.zeros(n, device="cuda", dtype=torch.bfloat16)
    ch = torch.tensor([[i, i, 1 << 16, 1, 1] for i in range(0, n, 1 << 16)], device="cuda")
    out.append(bench_mem("adam", lambda: ext().adam_segments(O, G, P, ch, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, 1.0),
                         n * (12 + 4 + 12 + 2), iters))
    return out


def bench_attention(iters, s=4096, b=1, G=32, hpg=1):
    """Causal attention at the 7B shape: native forward / backward vs PyTorch SDPA (library)."""
    from elasticmegatron_b200.ops.functional import _sdpa_attention
    from elasticmegatron_b200.ops.native import ext

    qkv = torch.randn(s, b, G, hpg + 2, 128, device="cuda").bfloat16()
    H = G * hpg
    flops_fwd = 4 * b * H * s * s * 128 / 2  # causal
    o, lse = ext().attn_fwd(qkv, hpg, True)
    dO = torch.randn_like(o)
    ms_f = timeit(lambda: ext().attn_fwd(qkv, hpg, True), iters)
    ms_b = timeit(lambda: ext().attn_bwd(dO, qkv, o, lse, hpg, True), iters)
    x = qkv.clone().requires_grad_(True)

    def sdpa_fb():
        y = _sdpa_attention(x, hpg)
        y.backward(dO)

    ms_sf = timeit(lambda: _sdpa_attention(qkv, hpg), iters)
    ms_sfb = timeit(sdpa_fb, iters)
    pk, _, src = peaks()
    return [{"op": "attn_fwd", "ms": ms_f, "tflops": flops_fwd / ms_f / 1e9, "frac": flops_fwd / ms_f / 1e9 / pk,
             "sdpa_ms": ms_sf, "sdpa_tflops": flops_fwd / ms_sf / 1e9, "peak": src},
            {"op": "attn_bwd", "ms": ms_b, "tflops": 2.5 * flops_fwd / ms_b / 1e9,
             "frac": 2.5 * flops_fwd / ms_b / 1e9 / pk, "sdpa_fwd_bwd_ms": ms_sfb, "native_fwd_bwd_ms": ms_f + ms_b,
             "peak": src}]


def bench_fused(m, n, k, iters):
    """gemm_rs / gemm_ag on one GPU, tp = 2 emulated with local buffers (see the module docstring)."""
    from elasticmegatron_b200.ops.native import ext

    pk, _, src = peaks()
    dev = "cuda"
    tp, R = 2, m // 2
    a = torch.randn(m, k, device=dev).bfloat16()
    w = torch.randn(n, k, device=dev).bfloat16()
    st = [torch.empty(tp * R * n, device=dev, dtype=torch.bfloat16) for _ in range(tp)]
    peers = torch.tensor([t.data_ptr() for t in st], dtype=torch.int64)
    rs = lambda: ext().gemm_rs(a, w, False, True, peers, 0, R)
    ms_rs = timeit(rs, iters)
    ms_red = timeit(lambda: ext().rs_reduce(st[0], tp, R, n), iters)
    # all-gather: own chunk 0 in place, chunk 1 pre-filled, its unit flags already at the epoch
    units_max = 1920
    local = torch.randn(m, k, device=dev).bfloat16()
    shard = local[:R].contiguous()
    other = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
    flags = [torch.zeros(tp * units_max, dtype=torch.int32, device=dev) for _ in range(tp)]
    epoch = 7
    flags[0][units_max:units_max + R // 32] = epoch
    fptr = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64)
    bptr = torch.tensor([local.data_ptr(), other.data_ptr()], dtype=torch.int64)
    claim = torch.zeros(1, dtype=torch.int32, device=dev)

    def ag():
        claim.zero_()
        return ext().gemm_ag(local, w, True, bptr, 0, R, claim, shard, fptr, epoch, units_max)

    y = ag()
    torch.cuda.synchronize()
    ok = torch.equal(other[:R], shard) and ext().gemm_error_flag() == 0
    ref = (local.float() @ w.float().t())
    err = float((y.float() - ref).abs().max() / ref.abs().max())
    ms_ag = timeit(ag, iters)
    ms_g = timeit(lambda: ext().gemm_tc(a, w, False, True), iters)
    fl = 2.0 * m * n * k
    return [{"op": "gemm_rs(emulated tp2)", "m": m, "n": n, "k": k, "ms": ms_rs, "tflops": fl / ms_rs / 1e9,
             "frac": fl / ms_rs / 1e9 / pk, "rs_reduce_ms": ms_red, "gemm_ms": ms_g, "peak": src},
            {"op": "gemm_ag(emulated tp2)", "m": m, "n": n, "k": k, "ms": ms_ag, "tflops": fl / ms_ag / 1e9,
             "frac": fl / ms_ag / 1e9 / pk, "gemm_ms": ms_g, "push_ok": bool(ok), "max_rel_err": err, "peak": src}]


def bench_reshard_local(iters, model="llama2-7b", layers=2):
    """K1 on ONE GPU: every rank's arenas of an 8-rank TP1*DP8 -> TP4*DP2 switch live on this device and all
    destination ranks' task tables run in one launch (a local strided copy: bytes read + written over the
    measured HBM copy bandwidth is its roofline)."""
    import numpy as np

    from elasticmegatron_b200.config import Args, TrainConfig, preset, set_args
    from elasticmegatron_b200.ops.native import ext
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.layout import rank_layout
    from elasticmegatron_b200.planner.plan import build_plan
    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine

    _, hbm, src = peaks()
    cfg = preset(model, num_layers=layers, max_tensor_parallel_size=8)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True)))
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)
    b = ParallelStrategy(world_size=8, tensor_model_parallel_size=4, pipeline_model_parallel_size=1)
    plan = build_plan(a, b, cfg, overlap_grad_reduce=True, ddp_bucket_size=None)
    bufs, addrs = [], {}
    for r in range(8):
        la, lb = rank_layout(cfg, a, r, True, None), rank_layout(cfg, b, r, True, None)
        t = [torch.randn(la.param_numel, device="cuda").bfloat16(), torch.rand(3, la.opt_numel, device="cuda"),
             torch.empty(lb.param_numel, device="cuda", dtype=torch.bfloat16),
             torch.empty(3, lb.opt_numel, device="cuda")]
        bufs.append(t)
        addrs[r] = tuple(x.data_ptr() for x in t)
    eng = NativeP2PEngine(mode="pull")
    tasks = np.concatenate([eng._tasks(plan, r, addrs, 2) for r in range(8)])
    tasks = tasks[np.argsort(-(tasks["rows"].astype(np.int64) * tasks["row_bytes"] * tasks["planes"]), kind="stable")]
    nbytes = int((tasks["rows"].astype(np.int64) * tasks["row_bytes"] * tasks["planes"]).sum())
    buf = torch.from_numpy(tasks.view(np.uint8).copy()).cuda()
    ms = timeit(lambda: ext().reshard_copy(buf, len(tasks), 0), iters)
    gbs = 2 * nbytes / ms / 1e6
    return [{"op": "reshard_copy(local, 8 ranks emulated)", "model": model, "layers": layers, "tasks": len(tasks),
             "bytes": nbytes, "ms": ms, "rw_gbs": gbs, "frac": gbs / hbm, "peak": src}]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "elementwise", "attention", "fused", "reshard", "all"])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--layout", default="fprop", help="fprop | dgrad | wgrad | tn | wgrad_bf16, or a comma list")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--baseline", action="store_true")
    ap.add_argument("--variant", type=int, default=0,
                    help="0 = variants 1 and 2; 1 one-SM tiles, 2 two-SM cluster tiles, 3 two-SM tiles without the "
                         "tail split, 9 two-SM tiles writing no output (measures the epilogue's share)")
    ap.add_argument("--variants", default=None, help="comma list of GEMM variants for 'all' (overrides --variant)")
    a = ap.parse_args()
    variants = [int(v) for v in a.variants.split(",")] if a.variants else ((1, 2) if a.variant == 0 else (a.variant,))
    res = []
    if a.what == "gemm":
        for lay in a.layout.split(","):
            res.append(bench_gemm(a.m, a.n, a.k, lay, a.iters, a.baseline, a.variant))
    if a.what == "fused":
        res += bench_fused(a.m, a.n, a.k, a.iters)
    if a.what == "reshard":
        res += bench_reshard_local(a.iters)
    if a.what == "all":
        # the Llama-2 7B training GEMMs at 4096 tokens per micro-batch
        for (m, n, k) in ((4096, 12288, 4096), (4096, 4096, 4096), (4096, 22016, 4096), (4096, 4096, 11008),
                          (4096, 32000, 4096)):
            for lay in ("fprop", "dgrad", "wgrad"):
                mm, nn, kk = (m, n, k) if lay == "fprop" else ((m, k, n) if lay == "dgrad" else (n, k, m))
                for j, var in enumerate(variants):
                    res.append(bench_gemm(mm, nn, kk, lay, a.iters, a.baseline and j == len(variants) - 1, var))
    if a.what in ("elementwise", "all"):
        res += bench_elementwise(a.iters)
    if a.what in ("attention", "all"):
        res += bench_attention(a.iters)
    for r in res:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
