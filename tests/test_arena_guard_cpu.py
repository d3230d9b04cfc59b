"""Guard words after every state arena (``EMB_ARENA_GUARD=1``): an out-of-bounds write is reported, in-bounds
work (training, switching, pool reuse) leaves them intact."""
import numpy as np
import pytest
import torch

from dist_utils import run_distributed
from test_elastic_cpu import STRATS, _train


def test_guard_catches_overrun(monkeypatch):
    from elasticmegatron_b200.runtime import memory

    monkeypatch.setenv("EMB_ARENA_GUARD", "1")
    pool = memory.ArenaPool(torch.device("cpu"))
    monkeypatch.setitem(memory._POOLS, "cpu-guard-test", pool)
    a = pool.alloc(1000, zero=True)
    assert a.used == 1000 and a.nbytes >= 1000 + memory.GUARD_BYTES
    v = a.view(torch.float32, (250,))
    v.fill_(1.0)  # the whole requested size
    memory.check_guards()
    with pytest.raises(AssertionError):
        a.view(torch.float32, (251,))  # views stop at the requested size
    a.raw[1000] = 0  # one byte past the end
    with pytest.raises(RuntimeError, match=f"arena {a.id}"):
        memory.check_guards("overrun")
    # a freed arena is not checked; reused for a smaller request its guard moves and is re-armed
    pool.free(a)
    memory.check_guards()
    b = pool.alloc(600)
    assert b is a and b.used == 600 and b.guard_intact()
    b.raw[599] = 7
    memory.check_guards()


def test_guard_off_by_default(monkeypatch):
    from elasticmegatron_b200.runtime import memory

    monkeypatch.delenv("EMB_ARENA_GUARD", raising=False)
    pool = memory.ArenaPool(torch.device("cpu"))
    a = pool.alloc(2 << 20)
    assert pool.guard == 0 and a.guard == 0 and a.nbytes == 2 << 20


def test_guards_intact_through_training_and_switches(monkeypatch):
    monkeypatch.setenv("EMB_ARENA_GUARD", "1")  # inherited by the spawned ranks
    base = run_distributed(_train, 2, [None] * 5, False, True, STRATS)
    sw = run_distributed(_train, 2, [None, 1, None, 2, 0], False, True, STRATS)
    np.testing.assert_allclose(base[0], sw[0], rtol=2e-6)
