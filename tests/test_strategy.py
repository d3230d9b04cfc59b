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
