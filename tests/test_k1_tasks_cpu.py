"""K1 task tables on the host (no GPU): splitting keeps every byte exactly once, and the task order is a
permutation that visits the peers round-robin from a rank-dependent start."""
import numpy as np


def _plan(tp_dst=1, pp_dst=8):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.plan import build_plan

    cfg = ModelConfig(num_layers=8, hidden_size=128, num_attention_heads=8, num_query_groups=4, ffn_hidden_size=192,
                      vocab_size=1000, params_dtype="bf16", max_tensor_parallel_size=4, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True, ddp_bucket_size=20000)))
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)
    b = ParallelStrategy(world_size=8, tensor_model_parallel_size=tp_dst, pipeline_model_parallel_size=pp_dst)
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


def _fake_addrs(plan, n=8):
    # every arena 1 TiB apart; a peer's mapping is just another base address
    return {r: tuple(int(np.uint64(1 << 40) * np.uint64(4 * r + j + 1)) for j in range(4)) for r in range(n)}


def test_validator_accepts_planned_tables_and_catches_corruption():
    import pytest

    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine
    from elasticmegatron_b200.transfer.validate import plan_regions, validate_tasks

    plan = _plan()
    addrs = _fake_addrs(plan)
    src, dst = plan_regions(plan, addrs, 2)
    assert len(src) == len(dst) == 16
    for mode in ("push", "pull"):
        eng = NativeP2PEngine(mode=mode, task_bytes=4096)
        for r in range(8):
            validate_tasks(eng._tasks(plan, r, addrs, 2), src, dst)
    t = NativeP2PEngine(mode="push", task_bytes=4096)._tasks(plan, 3, addrs, 2)
    assert len(t) > 10
    # a destination moved past the end of its arena
    bad = t.copy()
    end = max(b + n for b, n, _ in dst if b <= int(bad["dst"][5]) < b + n)
    bad["dst"][5] = end - int(bad["row_bytes"][5]) // 2
    with pytest.raises(ValueError, match="task 5: dst"):
        validate_tasks(bad, src, dst)
    # a source read from an address no arena covers
    bad = t.copy()
    bad["src"][2] = 16
    with pytest.raises(ValueError, match="task 2: src"):
        validate_tasks(bad, src, dst)
    # one extra row on a multi-row task (TP changes move 2-D boxes) runs past its arena
    plan = _plan(tp_dst=4, pp_dst=1)
    addrs = _fake_addrs(plan)
    src, dst = plan_regions(plan, addrs, 2)
    t = NativeP2PEngine(mode="push", task_bytes=1 << 20)._tasks(plan, 0, addrs, 2)
    validate_tasks(t, src, dst)
    multi = int(np.flatnonzero(t["rows"] > 1)[0])
    bad = t.copy()
    bad["rows"][multi] += 10 ** 6
    with pytest.raises(ValueError, match=f"task {multi}: dst"):
        validate_tasks(bad, src, dst)
    # two tasks writing the same bytes
    dup = np.concatenate([t, t[7:8]])
    with pytest.raises(ValueError, match="both write destination byte"):
        validate_tasks(dup, src, dst)
    # an empty task
    bad = t.copy()
    bad["rows"][0] = 0
    with pytest.raises(ValueError, match="task 0: empty"):
        validate_tasks(bad, src, dst)


def test_all_ranks_writes_are_disjoint():
    """The union over ranks of the push tables writes every destination byte at most once."""
    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine
    from elasticmegatron_b200.transfer.validate import plan_regions, validate_tasks

    for tp, pp in ((1, 8), (4, 1), (2, 2)):
        plan = _plan(tp, pp)
        addrs = _fake_addrs(plan)
        eng = NativeP2PEngine(mode="push", task_bytes=1 << 16)
        every = np.concatenate([eng._tasks(plan, r, addrs, 2) for r in range(8)])
        validate_tasks(every, *plan_regions(plan, addrs, 2))
