"""Inter-process elasticity agent: start a successor job, agree on the hand-off iteration, accept node triggers.

The reference drives inter-process scaling from a Megatron training loop with a helper module
(tools/agent/env_utils.py): it spawns replacement ``torchrun`` jobs with environment flags
(``_start_new_megatron_proc`` :214-323), signals readiness through a POSIX shared-memory byte
(``ready-flag shm`` :68-81) that the old job's rank 0 broadcasts to its peers
(examples/inter_process/training_011.py:103-119), and can ask another node to join through a TCP listener
that launches the demo script there (tools/agent/listening_add_nodes_multi.py:9-30, ``trigger_new_node``
env_utils.py:88-95).

Here the same three roles are small, testable pieces with bounded waits:

* :func:`spawn_successor` - start the new job (any command line, usually ``torchrun``) with the hand-off
  rendezvous in its environment (``EMB_ELASTIC_ROLE=successor``, ``EMB_HANDOFF_ROOT``, ``EMB_HANDOFF_TAG``);
* :func:`mark_ready` / :func:`poll_ready` / :func:`ready_consensus` - the successor marks itself ready (its
  process group and model exist) with an atomically created file; the old job checks it once per iteration,
  rank 0 reads and the decision is broadcast over the old job's host group, so every old rank hands off at the
  same iteration;
* :class:`NodeListener` / :func:`trigger_node` - a TCP listener that, on a JSON request, launches a command
  with the given environment (how a new node is told to start its part of the successor job).

State export / adoption itself is ``runtime/interprocess.py``.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import threading
import time
from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

ROLE_ENV = "EMB_ELASTIC_ROLE"
ROOT_ENV = "EMB_HANDOFF_ROOT"
TAG_ENV = "EMB_HANDOFF_TAG"


def role() -> str:
    """``"successor"`` inside a job started by :func:`spawn_successor`, else ``"primary"``."""
    return os.environ.get(ROLE_ENV, "primary")


def handoff_location() -> Optional[tuple]:
    root, tag = os.environ.get(ROOT_ENV), os.environ.get(TAG_ENV)
    return (root, tag) if root and tag else None


def spawn_successor(cmd: Sequence[str], root: str, tag: str, env: Optional[Dict[str, str]] = None,
                    log_path: Optional[str] = None, cwd: Optional[str] = None) -> subprocess.Popen:
    """Start the successor job (reference: env_utils.py:214-323).  The caller keeps the handle and, if it
    outlives the successor, reaps it; nothing is killed by pattern."""
    e = dict(os.environ)
    # the successor is its own job: never inherit the launcher's rank variables
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
              "TORCHELASTIC_RUN_ID", "TORCHELASTIC_RESTART_COUNT", "TORCHELASTIC_MAX_RESTARTS"):
        e.pop(k, None)
    e.update(env or {})
    e[ROLE_ENV] = "successor"
    e[ROOT_ENV] = root
    e[TAG_ENV] = tag
    os.makedirs(os.path.join(root, tag), exist_ok=True)
    out = open(log_path, "ab") if log_path else subprocess.DEVNULL
    try:
        return subprocess.Popen(list(cmd), env=e, stdout=out, stderr=subprocess.STDOUT, cwd=cwd,
                                start_new_session=True)
    finally:
        if log_path:
            out.close()


def mark_ready(root: str, tag: str, rank: int) -> None:
    """Successor rank ``rank`` is ready to adopt state (atomic create; idempotent)."""
    d = os.path.join(root, tag)
    os.makedirs(d, exist_ok=True)
    tmp = os.path.join(d, f".ready_{rank}.{os.getpid()}")
    with open(tmp, "w") as f:
        f.write(str(time.time()))
    os.replace(tmp, os.path.join(d, f"ready_{rank}"))


def poll_ready(root: str, tag: str, n: int) -> bool:
    """True when ``n`` successor ranks have marked themselves ready (non-blocking)."""
    d = os.path.join(root, tag)
    if not os.path.isdir(d):
        return False
    return sum(1 for f in os.listdir(d) if f.startswith("ready_")) >= n


def ready_consensus(root: str, tag: str, n: int, group=None) -> bool:
    """Collective over ``group`` (a gloo group of the old job; default: all ranks): its first rank polls and
    broadcasts the answer, so every old rank hands off at the same iteration."""
    if not dist.is_initialized():
        return poll_ready(root, tag, n)
    if group is None:
        from ..parallel.process_groups import ProcessGroupPool

        group = ProcessGroupPool.get(list(range(dist.get_world_size())), "gloo")
    src = dist.get_global_rank(group, 0)
    flag = torch.tensor([int(poll_ready(root, tag, n)) if dist.get_rank() == src else 0], dtype=torch.int64)
    dist.broadcast(flag, src=src, group=group)
    return bool(flag.item())


def wait_ready(root: str, tag: str, n: int, timeout: float = 600.0) -> None:
    t0 = time.time()
    while not poll_ready(root, tag, n):
        if time.time() - t0 > timeout:
            raise TimeoutError(f"successor did not become ready within {timeout}s")
        time.sleep(0.05)


class NodeListener:
    """TCP listener that launches a command per request (reference: listening_add_nodes_multi.py:9-30).

    A request is one JSON object ``{"cmd": [...], "env": {...}, "cwd": ...}`` terminated by a newline; the
    reply is ``{"ok": true, "pid": N}`` or ``{"ok": false, "error": ...}``.  ``allowed`` restricts the first
    argument of the command (default: the Python interpreter and ``torchrun``), since the listener runs
    whatever it is sent.
    """

    def __init__(self, host: str = "127.0.0.1", port: int = 0, allowed: Optional[List[str]] = None,
                 log_dir: Optional[str] = None):
        import sys

        self.allowed = allowed if allowed is not None else [sys.executable, "python", "python3", "torchrun"]
        self.log_dir = log_dir
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(8)
        self.sock.settimeout(0.2)
        self.address = self.sock.getsockname()
        self.launched: List[subprocess.Popen] = []
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._serve, daemon=True)

    def start(self) -> "NodeListener":
        self._thread.start()
        return self

    def _serve(self):
        while not self._stop.is_set():
            try:
                conn, _ = self.sock.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            with conn:
                conn.settimeout(5.0)
                try:
                    data = b""
                    while not data.endswith(b"\n") and len(data) < (1 << 20):
                        chunk = conn.recv(65536)
                        if not chunk:
                            break
                        data += chunk
                    req = json.loads(data.decode())
                    cmd = [str(x) for x in req["cmd"]]
                    if not cmd or cmd[0] not in self.allowed:
                        raise PermissionError(f"command {cmd[:1]} not allowed")
                    env = dict(os.environ)
                    env.update({str(k): str(v) for k, v in req.get("env", {}).items()})
                    log = open(os.path.join(self.log_dir, f"node_{len(self.launched)}.log"), "ab") \
                        if self.log_dir else subprocess.DEVNULL
                    p = subprocess.Popen(cmd, env=env, cwd=req.get("cwd"), stdout=log, stderr=subprocess.STDOUT,
                                         start_new_session=True)
                    if self.log_dir:
                        log.close()
                    self.launched.append(p)
                    reply = {"ok": True, "pid": p.pid}
                except Exception as e:  # reply with the error, keep serving
                    reply = {"ok": False, "error": repr(e)}
                try:
                    conn.sendall((json.dumps(reply) + "\n").encode())
                except OSError:
                    pass

    def close(self, wait: float = 10.0) -> None:
        self._stop.set()
        self._thread.join(timeout=2.0)
        self.sock.close()
        for p in self.launched:
            try:
                p.wait(timeout=wait)
            except subprocess.TimeoutExpired:
                p.terminate()


def trigger_node(host: str, port: int, cmd: Sequence[str], env: Optional[Dict[str, str]] = None,
                 cwd: Optional[str] = None, timeout: float = 10.0) -> Dict:
    """Ask the listener at ``host:port`` to start ``cmd`` (reference: env_utils.py:88-95)."""
    with socket.create_connection((host, port), timeout=timeout) as s:
        s.sendall((json.dumps({"cmd": list(cmd), "env": env or {}, "cwd": cwd}) + "\n").encode())
        data = b""
        while not data.endswith(b"\n"):
            chunk = s.recv(65536)
            if not chunk:
                break
            data += chunk
    return json.loads(data.decode())
