"""K1 task tables on the host (no GPU): splitting keeps every byte exactly once, and the task order is a
permutation that visits the peers round-robin from a rank-dependent start."""
import numpy as np


def _plan():
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.plan import build_plan

    cfg = ModelConfig(num_layers=8, hidden_size=128, num_attention_heads=8, num_query_groups=4, ffn_hidden_size=192,
                      vocab_size=1000, params_dtype="bf16", max_tensor_parallel_size=4, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True, ddp_bucket_size=20000)))
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)
    b = ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=8)
    return build_plan(a, b, cfg)


def _bytes(tasks):
    return int((tasks["rows"].astype(np.int64) * tasks["row_bytes"] * tasks["planes"]).sum())


def test_tasks_cover_the_plan_and_rotate_over_peers():
    from elasticmegatron_b200.planner.plan import KIND_OPT
    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine

    plan = _plan()
    d = plan.desc
    addrs = {r: tuple(np.uint64(1 << 40) * np.uint64(4 * r + j + 1) for j in range(4)) for r in range(8)}
    for mode in ("push", "pull"):
        for task_bytes in (4096, 1 << 20):
            eng = NativeP2PEngine(mode=mode, task_bytes=task_bytes)
            for r in range(8):
                t = eng._tasks(plan, r, addrs, 2)
                mine = d[(d["src_rank"] if mode == "push" else d["dst_rank"]) == r]
                el = np.where(mine["kind"] == KIND_OPT, 12, 2)
                assert _bytes(t) == int((mine["rows"] * mine["cols"] * el).sum())
                single = (t["rows"] == 1) | (t["row_bytes"].astype(np.int64) * t["planes"] > task_bytes)
                assert (single | (t["row_bytes"].astype(np.int64) * t["rows"] * t["planes"] <= task_bytes)).all()
                # peer of each task, recovered from its remote address range
                addr = t["dst"] if mode == "push" else t["src"]
                peer = ((addr.astype(np.uint64) >> np.uint64(40)).astype(np.int64) - 1) // 4
                first = [int(p) for p in peer[: len(set(peer.tolist()))]]
                others = [p for p in sorted(set(peer.tolist()))]
                rot = sorted(others, key=lambda p: (p - r - 1) % 8)
                assert first == rot, (mode, r, first, rot)
