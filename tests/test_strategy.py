"""ParallelStrategy derivations and rank meshes (reference: megatron_manager/parallel_strategy.py,
rank_generator.py)."""
import pytest

from elasticmegatron_b200.config import Args, ModelConfig, set_args
from elasticmegatron_b200.parallel.rank_generator import RankGenerator
from elasticmegatron_b200.parallel.strategy import ParallelStrategy


@pytest.fixture(autouse=True)
def _args():
    set_args(Args(model=ModelConfig(num_layers=8, num_experts=8)))
    yield


def test_rank_generator_megatron_order():
    g = RankGenerator(tp=2, ep=1, dp=2, pp=2, cp=1)
    assert g.get_ranks("tp") == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert g.get_ranks("dp") == [[0, 2], [1, 3], [4, 6], [5, 7]]
    assert g.get_ranks("pp") == [[0, 4], [1, 5], [2, 6], [3, 7]]
    assert g.get_ranks("tp-pp") == [[0, 1, 4, 5], [2, 3, 6, 7]]
    g = RankGenerator(tp=2, ep=1, dp=2, pp=1, cp=2)
    assert g.get_ranks("cp") == [[0, 2], [1, 3], [4, 6], [5, 7]]
    assert g.get_ranks("cp-dp") == [[0, 2, 4, 6], [1, 3, 5, 7]]


def test_strategy_derivations():
    s = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=2,
                         expert_model_parallel_size=2, expert_tensor_parallel_size=1)
    assert s.data_parallel_size == 2
    assert s.sequence_parallel is True
    assert s.expert_data_parallel_size == 2
    assert s.transformer_layer_num_per_stage == 4
    assert s.expert_num_per_ep_rank == 4
    s1 = ParallelStrategy(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                          expert_tensor_parallel_size=1)
    assert s1.sequence_parallel is False and s1.data_parallel_size == 4


def test_sp_requires_tp():
    with pytest.raises(ValueError):
        ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                         sequence_parallel=True, expert_tensor_parallel_size=1)


def test_every_rank_has_unique_coords():
    for tp, pp, cp in [(1, 1, 1), (2, 2, 1), (2, 1, 2), (4, 2, 1), (1, 8, 1), (8, 1, 1)]:
        s = ParallelStrategy(world_size=8, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp,
                             context_parallel_size=cp, expert_tensor_parallel_size=1,
                             sequence_parallel=tp > 1)
        seen = set()
        for r in range(8):
            c = s.coords(r)
            key = (c["tp"], c["cp"], c["dp"], c["pp"])
            assert key not in seen
            seen.add(key)
            assert s.rank_of(tp=c["tp"], cp=c["cp"], dp=c["dp"], pp=c["pp"]) == r


def test_group_zero_classification():
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                         num_distributed_optimizer_instances=2, expert_tensor_parallel_size=1)
    b = ParallelStrategy(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                         num_distributed_optimizer_instances=1, expert_tensor_parallel_size=1)
    assert ParallelStrategy.is_redundant_backup(a, b) is False
    assert ParallelStrategy.is_redundant_backup(b, a) is True
    c = ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                         expert_tensor_parallel_size=1)
    assert ParallelStrategy.is_redundant_backup(b, c) is None
    with pytest.raises(ValueError):
        ParallelStrategy.is_redundant_backup(a, a)


def test_identity_includes_sp():
    set_args(Args(model=ModelConfig(num_layers=8)))
    a = ParallelStrategy(world_size=2, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                         sequence_parallel=True, expert_tensor_parallel_size=1)
    b = ParallelStrategy(world_size=2, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                         sequence_parallel=False, expert_tensor_parallel_size=1)
    assert a != b and a.layout_key() == b.layout_key()


def test_parse_round_trip():
    from elasticmegatron_b200.config import Args, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy as P

    set_args(Args())  # a dense model (with experts, ETP must be given as etp1 when TP > 1)

    for spec in ("ws8", "ws2-tp2", "ws4-tp2-nosp", "ws8-tp2-pp2-cp1-dp2-ep1-etp2-inst1-sp", "ws8-ep4-inst2",
                 "ws8-tp2-cp2-pp2"):
        s = P.parse(spec)
        assert P.parse(str(s)) == s and P.from_any(str(s)) == s
    assert P.parse("ws4-tp2").sequence_parallel and not P.parse("ws4-tp2-nosp").sequence_parallel
    import pytest

    with pytest.raises(ValueError):
        P.parse("tp2")
    with pytest.raises(ValueError):
        P.parse("ws4-xx2")


def _divisors(n):
    return [d for d in range(1, n + 1) if n % d == 0]


def _oracle_groups(sizes, order, token):
    """Megatron's documented mesh: rank = sum(coord * stride) with the first axis of ``order`` fastest; a group
    of ``token`` is every rank that shares the coordinates of the axes the token does not name.  Ranks inside a
    group and groups (by their lowest rank) come in ascending order."""
    named = set(token.split("-"))
    world = 1
    for ax in order:
        world *= sizes[ax]
    groups = {}
    for r in range(world):
        rest, key = r, []
        for ax in order:
            rest, c = divmod(rest, sizes[ax])
            if ax not in named:
                key.append((ax, c))
        groups.setdefault(tuple(key), []).append(r)
    return sorted(groups.values())


def _tokens(axes):
    from itertools import combinations

    return ["-".join(c) for k in range(1, len(axes) + 1) for c in combinations(axes, k)]


def test_rank_meshes_all_factorizations_of_1_2_4_8():
    """Dense (tp-cp-dp-pp) and expert (etp-ep-edp-pp) meshes of every strategy on 1, 2, 4 and 8 GPUs, every
    group token, against the oracle above."""
    order = ["tp", "cp", "ep", "dp", "pp"]
    n = 0
    for ws in (1, 2, 4, 8):
        for tp in _divisors(ws):
            for cp in _divisors(ws // tp):
                for pp in _divisors(ws // (tp * cp)):
                    dp = ws // (tp * cp * pp)
                    s = ParallelStrategy(world_size=ws, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp,
                                         context_parallel_size=cp, expert_tensor_parallel_size=1,
                                         sequence_parallel=tp > 1,
                                         expert_model_parallel_size=max(e for e in _divisors(ws // pp) if 8 % e == 0))
                    dense = dict(tp=tp, cp=cp, ep=1, dp=dp, pp=pp)
                    for tok in _tokens(["tp", "cp", "dp", "pp"]):
                        assert s.all_groups(tok) == _oracle_groups(dense, order, tok), (ws, tp, cp, pp, tok)
                        n += 1
                    ep = s.expert_model_parallel_size
                    expert = dict(tp=1, cp=1, ep=ep, dp=ws // (ep * pp), pp=pp)
                    for tok in _tokens(["tp", "ep", "dp", "pp"]):
                        assert s.all_groups(tok, True) == _oracle_groups(expert, order, tok), (ws, ep, pp, tok)
                    # the expert mesh with ETP > 1 (no MoE resharding support, but the mesh itself)
                    for etp in _divisors(ws // pp):
                        for ep2 in _divisors(ws // (pp * etp)):
                            sizes = dict(tp=etp, cp=1, ep=ep2, dp=ws // (etp * ep2 * pp), pp=pp)
                            g = RankGenerator(tp=etp, ep=ep2, dp=sizes["dp"], pp=pp, cp=1)
                            for tok in ("tp", "ep", "dp", "pp", "tp-ep", "ep-dp", "tp-ep-pp"):
                                assert g.get_ranks(tok) == _oracle_groups(sizes, order, tok), (ws, etp, ep2, pp, tok)
    assert n > 300
