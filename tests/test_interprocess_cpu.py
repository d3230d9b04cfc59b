"""Inter-process hand-off on CPU/gloo: a 2-rank job exports its state in place, a separate 1-rank job adopts it
(pulling its own layout straight out of the old processes' shared memory) and continues training; the loss
equals an in-process reshard of the same schedule."""
import tempfile

import numpy as np
import torch.multiprocessing as mp

from dist_utils import _entry, free_port, run_distributed
from test_elastic_cpu import STRATS, _setup


def _continuous(rank, world):
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    S = [ParallelStrategy(**s) for s in STRATS]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(STRATS, training_state=ts, engine="torch")
    it = mgr.build_iterators(0)[0]
    train_step(ts, it)
    train_step(ts, it)
    ts = mgr.reshard(STRATS[3])
    if ts is None:
        return None
    return train_step(ts, mgr.build_iterators(16)[0])["loss"]


def _old_job(rank, world, root):
    from elasticmegatron_b200.config import get_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import export_state, wait_for_acks
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    ts = TrainingState(ParallelStrategy(**STRATS[0]))
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    train_step(ts, it)
    train_step(ts, it)
    get_args().iteration, get_args().consumed_train_samples = 2, 16
    export_state(ts, root, "scale_down")
    wait_for_acks(root, "scale_down", 1, timeout=120)
    return True


def _new_job(rank, world, root):
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import ack, adopt, import_records
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    ts = TrainingState(ParallelStrategy(**STRATS[3]))
    recs = import_records(root, "scale_down", old_world=2, timeout=120)
    info = adopt(ts, recs)
    ack(root, "scale_down", rank)
    assert info["iteration"] == 2
    return train_step(ts, DataloaderState.build_iterators(ts, info["consumed_train_samples"])[0])["loss"]


def test_scale_down_handoff_matches_in_process_reshard():
    ref = run_distributed(_continuous, 2)[0]
    root = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    old = [ctx.Process(target=_entry, args=(r, 2, port, _old_job, (root,), q)) for r in range(2)]
    for p in old:
        p.start()
    new = run_distributed(_new_job, 1, root)
    res = [q.get(timeout=120) for _ in range(2)]
    for p in old:
        p.join(timeout=60)
    assert all(r[1] == "ok" for r in res), res
    np.testing.assert_allclose(new[0], ref, rtol=1e-6)


def _continuous_up(rank, world):
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    order = [STRATS[3], STRATS[1]]
    S = [ParallelStrategy(**s) for s in order]
    create_all_groups(S)
    ts = TrainingState(S[0]) if rank == 0 else None
    if ts is not None:
        ts.init_weights(0)
    mgr = ElasticMegatronManager(order, training_state=ts, engine="torch")
    if ts is not None:
        it = mgr.build_iterators(0)[0]
        train_step(ts, it)
        train_step(ts, it)
    ts = mgr.reshard(STRATS[1])
    return train_step(ts, mgr.build_iterators(16)[0])["loss"]


def _old_job_up(rank, world, root):
    from elasticmegatron_b200.config import get_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import export_state, wait_for_acks
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    ts = TrainingState(ParallelStrategy(**STRATS[3]))
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    train_step(ts, it)
    train_step(ts, it)
    get_args().iteration, get_args().consumed_train_samples = 2, 16
    export_state(ts, root, "scale_up")
    wait_for_acks(root, "scale_up", 2, timeout=120)
    return True


def _new_job_up(rank, world, root):
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import ack, adopt, import_records
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    s = ParallelStrategy(**STRATS[1])
    create_all_groups([s])
    ts = TrainingState(s)
    recs = import_records(root, "scale_up", old_world=1, timeout=120)
    info = adopt(ts, recs)
    ack(root, "scale_up", rank)
    assert info["iteration"] == 2
    return train_step(ts, DataloaderState.build_iterators(ts, info["consumed_train_samples"])[0])["loss"]


def test_scale_up_handoff_matches_in_process_reshard():
    """1 rank -> a new 2-rank TP2 job: the successor pulls its TP shards out of the single old process."""
    ref = run_distributed(_continuous_up, 2)[0]
    root = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    old = ctx.Process(target=_entry, args=(0, 1, free_port(), _old_job_up, (root,), q))
    old.start()
    new = run_distributed(_new_job_up, 2, root)
    res = q.get(timeout=120)
    old.join(timeout=60)
    assert res[1] == "ok", res
    np.testing.assert_allclose(new[0], ref, rtol=1e-6)
    np.testing.assert_allclose(new[1], ref, rtol=1e-6)
