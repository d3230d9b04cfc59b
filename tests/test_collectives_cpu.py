"""Host-side collective helpers on gloo ranks.

* the tensor/sequence-parallel mappings of ``ops/functional.py`` (forward and backward of each against the
  single-process math of the full tensor);
* the opt-in ``torch.distributed`` default-group patch (collectives without ``group=`` act on the active
  strategy's world);
* ``gather_from_rank`` inverts ``scatter_to_rank`` for every rank of a TP x PP x DP layout.
"""
import torch

from tests.dist_utils import run_distributed


def _mappings(rank, world):
    import torch.distributed as dist

    from elasticmegatron_b200.ops import functional as F_

    g = dist.group.WORLD
    full = torch.arange(world * 3 * 4, dtype=torch.float32).reshape(world * 3, 4)
    mine = full[rank * 3:(rank + 1) * 3]
    # every rank's upstream gradient differs, so sums over ranks are visible
    dys = [torch.full((world * 3, 4), float(r + 1)) for r in range(world)]
    out = {}

    x = mine.clone().requires_grad_()
    y = F_.gather_from_sp(x, g)
    y.backward(dys[rank])
    out["gather_fwd"] = torch.equal(y, full)
    out["gather_bwd"] = torch.equal(x.grad, sum(d[rank * 3:(rank + 1) * 3] for d in dys))

    x = full.clone().requires_grad_()
    y = F_.scatter_to_sp(x, g)
    y.backward(dys[rank][:3])
    out["scatter_fwd"] = torch.equal(y, mine)
    out["scatter_bwd"] = torch.equal(x.grad, torch.cat([d[:3] for d in dys]))

    x = (full * (rank + 1)).requires_grad_()
    y = F_.reduce_scatter_to_sp(x, g)
    y.backward(dys[rank][:3])
    tot = sum(full * (r + 1) for r in range(world))
    out["rs_fwd"] = torch.equal(y, tot[rank * 3:(rank + 1) * 3])
    out["rs_bwd"] = torch.equal(x.grad, torch.cat([d[:3] for d in dys]))

    x = full.clone().requires_grad_()
    y = F_.copy_to_tp(x, g)
    y.backward(dys[rank].clone())  # the backward all-reduces the incoming gradient in place
    out["copy_fwd"] = torch.equal(y, full)
    out["copy_bwd"] = torch.equal(x.grad, sum(dys))

    x = (full * (rank + 1)).requires_grad_()
    y = F_.reduce_from_tp(x, g)
    y.backward(dys[rank])
    out["reduce_fwd"] = torch.equal(y, tot)
    out["reduce_bwd"] = torch.equal(x.grad, dys[rank])
    return out


def test_tp_sp_mappings_forward_backward():
    for res in run_distributed(_mappings, 2):
        assert all(res.values()), res


def _patched(rank, world):
    import torch.distributed as dist

    from elasticmegatron_b200.parallel import process_groups as pg

    singles = [dist.new_group([r]) for r in range(world)]
    out = {}
    original = dist.all_reduce
    pg.patch_torch_distributed()
    out["patched"] = dist.all_reduce is not original
    try:
        t = torch.ones(1)
        dist.all_reduce(t)  # no active world: all launched ranks
        out["unset"] = t.item()
        with pg.with_world_group(singles[rank]):
            assert pg.get_world_group() is singles[rank]
            t = torch.ones(1)
            dist.all_reduce(t)  # acts on this rank's one-rank world
            out["active"] = t.item()
            t = torch.ones(1)
            dist.all_reduce(t, group=dist.group.WORLD)  # an explicit group wins
            out["explicit"] = t.item()
        out["restored"] = pg.get_world_group() is None
    finally:
        pg.unpatch_torch_distributed()
    out["unpatched"] = dist.all_reduce is original
    return out


def test_default_group_patch():
    for res in run_distributed(_patched, 2):
        assert res == {"patched": True, "unset": 2.0, "active": 1.0, "explicit": 2.0, "restored": True, "unpatched": True}, res


def test_gather_inverts_scatter():
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.layout import rank_layout, virtual_params
    from elasticmegatron_b200.planner.materialize import gather_from_rank, init_global_params, scatter_to_rank

    cfg = ModelConfig(num_layers=4, hidden_size=64, num_attention_heads=8, num_query_groups=4, ffn_hidden_size=96,
                      vocab_size=300, params_dtype="fp32", max_tensor_parallel_size=4, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True)))
    s = ParallelStrategy.parse("ws8-tp2-pp2")
    g = init_global_params(cfg, seed=3)
    gen = torch.Generator().manual_seed(4)
    og = {k: torch.stack([v, torch.rand(v.shape, generator=gen), torch.rand(v.shape, generator=gen)])
          for k, v in g.items()}
    outp = {k: torch.full_like(v, float("nan")) for k, v in g.items()}
    outo = {k: torch.full_like(v, float("nan")) for k, v in og.items()}
    for r in range(s.world_size):
        rl = rank_layout(cfg, s, r, True, None)
        P = torch.empty(rl.param_numel)
        O = torch.empty(3, rl.opt_numel)
        scatter_to_rank(cfg, s, r, g, P, O, og, True, None)
        gather_from_rank(cfg, s, r, outp, outo, P, O, True, None)
    for vp in virtual_params(cfg):
        assert torch.equal(outp[vp.index], g[vp.index]), vp
        assert torch.equal(outo[vp.index], og[vp.index]), vp


def _nvls_fallback(rank, world):
    import os

    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.parallel import nvls

    out = {}
    for v, want in (("1", "auto"), ("nvls", "nvls"), ("p2p", "p2p"), ("0", "off"), ("nccl", "off")):
        os.environ["EMB_NVLS"] = v
        out[v] = nvls.mode() == want
    os.environ["EMB_NVLS"] = "1"
    # host tensors on a gloo group take the library all-reduce (the symmetric reducers are CUDA-only)
    x = torch.arange(6, dtype=torch.float32) * (rank + 1)
    ref = x.clone()
    dist.all_reduce(ref)
    nvls.all_reduce_(x, dist.group.WORLD)
    out["sum"] = bool(torch.equal(x, ref))
    out["no_reducer"] = len(nvls._CACHE) == 0
    return out


def test_symmetric_all_reduce_host_fallback():
    """EMB_NVLS parsing, and the NCCL / gloo fallback for tensors the symmetric reducers do not take."""
    for r in run_distributed(_nvls_fallback, 2):
        assert all(r.values()), r
