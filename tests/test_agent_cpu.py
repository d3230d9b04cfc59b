"""Inter-process agent pieces and the two example programs, on CPU (gloo ranks, torchrun subprocesses)."""
import json
import os
import re
import subprocess
import sys

import pytest

from dist_utils import free_port

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ready_flags(tmp_path):
    from elasticmegatron_b200.runtime import agent

    root, tag = str(tmp_path), "t"
    assert not agent.poll_ready(root, tag, 1)
    agent.mark_ready(root, tag, 0)
    agent.mark_ready(root, tag, 0)  # idempotent
    assert agent.poll_ready(root, tag, 1) and not agent.poll_ready(root, tag, 2)
    agent.mark_ready(root, tag, 1)
    agent.wait_ready(root, tag, 2, timeout=1.0)
    with pytest.raises(TimeoutError):
        agent.wait_ready(root, tag, 3, timeout=0.2)


def test_node_listener_launches_allowed_commands(tmp_path):
    from elasticmegatron_b200.runtime import agent

    out = tmp_path / "started.txt"
    lst = agent.NodeListener(log_dir=str(tmp_path)).start()
    try:
        host, port = lst.address
        r = agent.trigger_node(host, port, [sys.executable, "-c",
                                            f"import os; open({str(out)!r}, 'w').write(os.environ['NEW_NODE'])"],
                               env={"NEW_NODE": "1"})
        assert r["ok"] and r["pid"] > 0
        r2 = agent.trigger_node(host, port, ["/bin/sh", "-c", "true"])
        assert not r2["ok"] and "not allowed" in r2["error"]
        lst.launched[0].wait(timeout=60)
    finally:
        lst.close()
    assert out.read_text() == "1"


def test_spawn_successor_environment(tmp_path):
    from elasticmegatron_b200.runtime import agent

    log = tmp_path / "succ.log"
    env_before = dict(os.environ)
    os.environ["RANK"] = "3"
    try:
        p = agent.spawn_successor([sys.executable, "-c", "import os; print(os.environ.get('RANK'), "
                                   "os.environ['EMB_ELASTIC_ROLE'], os.environ['EMB_HANDOFF_TAG'])"],
                                  str(tmp_path), "tg", log_path=str(log))
        assert p.wait(timeout=60) == 0
    finally:
        os.environ.clear()
        os.environ.update(env_before)
    assert log.read_text().split() == ["None", "successor", "tg"]


_LOSS = re.compile(r"iteration\s+(\d+)/\s*\d+ \|.*lm loss: ([0-9.E+-]+)")


def _losses(text):
    return {int(m.group(1)): float(m.group(2)) for m in _LOSS.finditer(text)}


def _torchrun(nproc, script, args, timeout=600):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", os.path.join(REPO, "examples", script)] + args
    env = dict(os.environ)
    env["PYTHONPATH"] = REPO + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout, cwd=REPO)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return r.stdout


def test_examples_handoff_matches_intra_process_switch(tmp_path):
    common = ["--cpu", "--layers", "2", "--seq-length", "64", "--train-iters", "6", "--global-batch-size", "8"]
    intra = _torchrun(2, "intra_process/train_elastic.py",
                      common + ["--strategies", "ws2,ws1", "--switch-every", "3", "--lr-warmup-iters", "0"])
    inter = _torchrun(2, "inter_process/train_handoff.py",
                      common + ["--strategy", "ws2", "--successor-strategy", "ws1", "--handoff-at", "3",
                                "--block-at-handoff", "--wait-successor", "--successor-port", str(free_port()),
                                "--handoff-root", str(tmp_path)])
    a, b = _losses(intra), _losses(inter)
    assert sorted(a) == sorted(b) == list(range(1, 7)), (intra[-2000:], inter[-2000:])
    for i in range(1, 7):
        assert abs(a[i] - b[i]) <= 1e-5 * abs(a[i]), (i, a[i], b[i])
    assert "successor exit code 0" in inter
    # structured lines: one per iteration (tokens/s/GPU, strategy) and one per switch (phases, link bytes)
    recs = [json.loads(ln) for ln in intra.splitlines() if ln.startswith('{"event"')]
    its = [r for r in recs if r["event"] == "iteration"]
    assert [r["iteration"] for r in its] == list(range(1, 7))
    assert [r["strategy"].split("-")[0] for r in its] == ["ws2"] * 3 + ["ws1"] * 3
    assert all(r["tokens_per_s_per_gpu"] > 0 for r in its)
    sw = [r for r in recs if r["event"] == "reshard"]
    assert len(sw) == 1 and (sw[0]["src"].split("-")[0], sw[0]["dst"].split("-")[0]) == ("ws2", "ws1")
    for k in ("build_ms", "plan_ms", "transfer_ms", "lr_ms", "release_ms", "total_ms"):
        assert sw[0][k] >= 0, k
    assert sw[0]["total_ms"] >= sw[0]["transfer_ms"]
    assert len(sw[0]["link_gb"]) == 2 and sw[0]["link_gb"][0][0] == 0 and sw[0]["max_egress_gb"] > 0


def test_handoff_chain_scale_down_and_up(tmp_path):
    """Three jobs: 2 ranks -> 1 rank -> 2 ranks (the 8 -> 4 -> 8 configuration in small), each adopting the
    previous job's state; the losses equal one job that switches at the same iterations."""
    common = ["--cpu", "--layers", "2", "--seq-length", "64", "--train-iters", "6", "--global-batch-size", "8"]
    intra = _torchrun(2, "intra_process/train_elastic.py",
                      common + ["--strategies", "ws2,ws1,ws2", "--switch-every", "2", "--lr-warmup-iters", "0"])
    inter = _torchrun(2, "inter_process/train_handoff.py",
                      common + ["--chain", "ws2,ws1,ws2", "--handoff-at", "2", "--block-at-handoff", "--wait-successor",
                                "--successor-port", str(free_port()), "--handoff-root", str(tmp_path)])
    a, b = _losses(intra), _losses(inter)
    assert sorted(a) == sorted(b) == list(range(1, 7)), (intra[-2000:], inter[-3000:])
    for i in range(1, 7):
        assert abs(a[i] - b[i]) <= 1e-5 * abs(a[i]), (i, a[i], b[i])
    assert inter.count("successor exit code 0") == 2
