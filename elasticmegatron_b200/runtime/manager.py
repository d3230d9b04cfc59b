"""``ElasticMegatronManager``: online switching between parallel strategies.

Public API kept from the reference (elastic_megatron/elastic_manager.py:31-265):

* ``ElasticMegatronManager.register(setup_model_and_optimizer_func, train_valid_test_datasets_provider)``
* ``ElasticMegatronManager(parallel_strategy_list, model, optimizer, opt_param_scheduler, ...)``
* ``reshard(new_parallel_strategy, logger=None, is_meta_device=False, save_ckpt=False) -> TrainingState | None``
* ``build_iterators()``, ``get_data_parallel_group(strategy)``, ``global_barrier_by_gloo()``,
  ``clear_meta_state(strategy)``.

A switch (reference call stack: elastic_manager.py:189-258):

1. build (lazily, cached per strategy) or rebuild the destination ``TrainingState``;
2. plan once per (src, dst) pair (``planner/plan.py``) - exact shard-to-shard ranges for fp32 master /
   exp_avg / exp_avg_sq *and* the parameters;
3. execute the plan with the selected engine (direct peer-memory kernel on GPUs, batched P2P otherwise);
   a Group-ZeRO instance-count change is the same plan (replica copies) instead of a separate code path;
4. copy LR / scheduler / step counters from rank 0 over the union group;
5. release the source state into the arena pool (no ``empty_cache``);
6. log one JSON line with device time (MAX over the union), bytes moved and the NVLink roofline fraction.
"""
from __future__ import annotations

import contextlib
import os
import logging
from typing import Callable, Dict, List, Optional, Union

import numpy as np
import torch
import torch.distributed as dist

from ..config import get_args
from ..parallel.process_groups import (ProcessGroupPool, create_all_groups, global_barrier_by_gloo,
                                       set_world_group)
from ..parallel.strategy import ParallelStrategy, union_ranks
from ..planner.plan import KIND_OPT, KIND_PARAM, build_plan
from ..utils.logging import log_json
from ..utils.timers import DeviceTimer, HostTimer, max_over_ranks, nvtx_range
from .data import DataloaderState
from .training_state import TrainingState

from ..utils.links import NVLINK_NOMINAL_GBS, measured_link_gbs


def default_setup_model_and_optimizer(strategy: ParallelStrategy, is_meta_device: bool = False) -> TrainingState:
    return TrainingState(strategy, is_meta_device=is_meta_device)


class ElasticMegatronManager:
    @classmethod
    def register(cls, setup_model_and_optimizer_func: Optional[Callable] = None,
                 train_valid_test_datasets_provider: Optional[Callable] = None) -> None:
        TrainingState.setup_model_and_optimizer_func = setup_model_and_optimizer_func
        DataloaderState.register(train_valid_test_datasets_provider)

    def __init__(self, parallel_strategy_list: List[Union[Dict, ParallelStrategy, str]], model=None, optimizer=None,
                 opt_param_scheduler=None, send_fn: Optional[Callable] = None, recv_fn: Optional[Callable] = None,
                 broadcast_fn: Optional[Callable] = None, use_p2p_to_collective: Optional[bool] = None,
                 training_state: Optional[TrainingState] = None, engine: Optional[str] = None,
                 prebuild_plans: Optional[bool] = None):
        """``send_fn`` / ``recv_fn`` / ``broadcast_fn`` / ``use_p2p_to_collective`` keep the reference's
        injectable communicator (elastic_manager.py:41-58): when any is given, switches run the reference's
        transfer schedule through those functions; otherwise ``engine`` picks the transfer engine
        ("native" peer-memory kernel on GPUs by default, "torch" batched P2P, "reference")."""
        self._rank = dist.get_rank() if dist.is_initialized() else 0
        self.strategies = [ParallelStrategy.from_any(s) for s in parallel_strategy_list]
        assert len(set(self.strategies)) == len(self.strategies), "duplicate strategies"
        backend = dist.get_backend() if dist.is_initialized() else "gloo"
        pairs = []
        if use_p2p_to_collective and dist.is_initialized():
            # P2P as a broadcast needs a group per rank pair; the reference builds all N(N-1)/2 of them up front
            # (distributed/elastic_process_group.py:235-245), collectively here like every other group
            n = dist.get_world_size()
            pairs = [(i, j) for i in range(n) for j in range(i + 1, n)]
        create_all_groups(self.strategies, backend, extra=pairs)
        if training_state is None and model is not None:
            training_state = model[0]._training_state
        self._states: Dict[ParallelStrategy, Optional[TrainingState]] = {s: None for s in self.strategies}
        self.current = self.strategies[0]
        if training_state is not None:
            assert training_state.strategy == self.strategies[0], "strategy 0 must match the live model"
            self._states[self.current] = training_state
        self._plans: Dict[tuple, object] = {}
        custom = any(x is not None for x in (send_fn, recv_fn, broadcast_fn, use_p2p_to_collective))
        if custom:
            from ..transfer.reference_engine import ReferenceAlgorithmEngine

            self.engine_name = "reference"
            self.engine = ReferenceAlgorithmEngine(send_fn, recv_fn, broadcast_fn, bool(use_p2p_to_collective))
        else:
            self.engine_name = engine or ("native" if torch.cuda.is_available() else "torch")
            self.engine = self._make_engine(self.engine_name)
        self.last_switch: Dict = {}
        self._warm_only = False
        set_world_group(ProcessGroupPool.get(self.current.ranks))
        self.memory_warnings = self._check_memory()
        # every declared switch's plan is host work that depends only on the two strategies: build them all now
        # (default for up to 8 strategies) so a switch's first occurrence does not pay for planning
        if prebuild_plans is None:
            prebuild_plans = len(self.strategies) <= 8 and os.environ.get("EMB_PREBUILD_PLANS", "1") != "0"
        self.plan_prebuild_ms = self.prebuild_plans() if prebuild_plans else 0.0

    def prebuild_plans(self) -> float:
        """Build the plans of all ordered pairs of declared strategies (host only); returns the time in ms."""
        import time

        t0 = time.perf_counter()
        for a in self.strategies:
            for b in self.strategies:
                if a != b:
                    self.plan(a, b)
        return (time.perf_counter() - t0) * 1e3

    def _check_memory(self) -> List[Dict]:
        """Warn (one JSON line each, never fail) about switches whose source and destination state cannot sit
        in this GPU's memory together (``planner/memory.py``)."""
        if not torch.cuda.is_available():
            return []
        try:
            from ..planner.memory import state_bytes

            cap = torch.cuda.get_device_properties(torch.cuda.current_device()).total_memory
            tc = get_args().train
            cfg = get_args().model
            mine = {s: state_bytes(cfg, s, self._rank, tc.overlap_grad_reduce, tc.ddp_bucket_size)["total"]
                    for s in self.strategies if self._rank < s.world_size}
            out = []
            for a in mine:
                for b in mine:
                    if a != b and mine[a] + mine[b] > 0.95 * cap:
                        w = {"src": str(a), "dst": str(b), "state_gb": (mine[a] + mine[b]) / 1e9, "device_gb": cap / 1e9}
                        out.append(w)
                        log_json("memory_warning", None, **w)
            return out
        except Exception:  # an estimate must never stop a job
            return []

    # ------------------------------------------------------------------ helpers
    def _make_engine(self, name: str):
        if name == "torch":
            from ..transfer.torch_engine import TorchP2PEngine

            return TorchP2PEngine()
        if name == "reference":
            from ..transfer.reference_engine import ReferenceAlgorithmEngine

            return ReferenceAlgorithmEngine()
        if name == "native":
            from ..transfer.native_engine import NativeP2PEngine

            return NativeP2PEngine()
        raise ValueError(name)

    @property
    def training_state(self) -> Optional[TrainingState]:
        return self._states.get(self.current)

    def state_for(self, strategy) -> Optional[TrainingState]:
        return self._states.get(ParallelStrategy.from_any(strategy))

    def plan(self, src: ParallelStrategy, dst: ParallelStrategy):
        key = (src.key(), dst.key())
        p = self._plans.get(key)
        if p is None:
            p = build_plan(src, dst)
            self._plans[key] = p
        return p

    def _get_or_build(self, s: ParallelStrategy, is_meta: bool) -> Optional[TrainingState]:
        if self._rank >= s.world_size:
            return None
        ts = self._states.get(s)
        if ts is None:
            fn = TrainingState.setup_model_and_optimizer_func or default_setup_model_and_optimizer
            ts = fn(s, is_meta_device=is_meta)
            self._states[s] = ts
        elif not is_meta:
            ts.rebuild()
        return ts

    # ------------------------------------------------------------------ API
    def build_iterators(self, consumed_samples: Optional[int] = None):
        ts = self.training_state
        if ts is None:
            return None, None, None
        if consumed_samples is None:
            consumed_samples = get_args().consumed_train_samples
        # consumed samples from rank 0 (reference: dataloader_state.py:135-141)
        t = torch.tensor([consumed_samples], dtype=torch.float64)
        if dist.is_initialized() and self.current.world_size > 1:
            dist.broadcast(t, src=0, group=ProcessGroupPool.get(self.current.ranks, "gloo"))
        return DataloaderState.build_iterators(ts, int(t.item()))

    def need_resharding(self, parallel_strategy) -> bool:
        """True when ``parallel_strategy`` differs from the current one (reference: megatron_state.py:151-156)."""
        return ParallelStrategy.from_any(parallel_strategy) != self.current

    def get_data_parallel_group(self, parallel_strategy):
        s = ParallelStrategy.from_any(parallel_strategy)
        if self._rank >= s.world_size:
            return None
        return ProcessGroupPool.get(s.get_ranks("dp"))

    @classmethod
    def global_barrier_by_gloo(cls):
        global_barrier_by_gloo()

    def clear_meta_state(self, parallel_strategy) -> None:
        s = ParallelStrategy.from_any(parallel_strategy)
        ts = self._states.get(s)
        if ts is not None:
            assert ts.is_meta_device
        self._states[s] = None

    def reshard(self, new_parallel_strategy, logger: Optional[logging.Logger] = None, is_meta_device: bool = False,
                save_ckpt: bool = False, ckpt_dir: Optional[str] = None) -> Optional[TrainingState]:
        """Switch to ``new_parallel_strategy``; returns this rank's state under it (None on idle ranks).

        ``logger`` receives the switch's JSON record (default: rank 0 prints it); ``save_ckpt`` writes Megatron
        checkpoints of both sides into ``<ckpt_dir>/before_reshard`` and ``<ckpt_dir>/after_reshard``."""
        # meta mode (or inside build_nccl_connection_context): build the destination's state and the switch's
        # mappings / task tables, move no data, and leave every live state alone - neither the source is
        # released nor a released state rebuilt (the reference turns release / rebuild into no-ops for its fake
        # transfers, elastic_manager.py:268-304)
        is_meta_device = is_meta_device or self._warm_only
        if is_meta_device and save_ckpt:
            raise ValueError("reshard: save_ckpt needs real tensors; a meta-device switch moves no data to save")
        dst_s = ParallelStrategy.from_any(new_parallel_strategy)
        assert dst_s in self._states, f"strategy {dst_s} was not declared at construction"
        src_s = self.current
        src = self._states.get(src_s)
        if save_ckpt and src is not None:
            from .checkpoint import save_checkpoint

            # the reference writes the two sides of a switch to before_reshard / after_reshard (its
            # convert-and-compare check reads both); ``ckpt_dir`` is the root that holds them
            save_checkpoint(src, os.path.join(ckpt_dir or ".", "before_reshard"))
        if dst_s == src_s:
            return src
        union = union_ranks(src_s, dst_s)
        if self._rank not in union:
            self.current = dst_s
            set_world_group(ProcessGroupPool.get(dst_s.ranks))
            return None
        ugroup = ProcessGroupPool.get(union)
        same_layout = src_s.layout_key() == dst_s.layout_key()
        # same layout (the strategies differ only in sequence parallelism): the destination takes over the
        # source's arenas - nothing is allocated and nothing moves
        adopt = same_layout and src is not None and not is_meta_device
        t_total = HostTimer(sync=False).__enter__()
        with HostTimer(sync=False) as t_build, nvtx_range("reshard/build"):
            dst = self._get_or_build(dst_s, is_meta_device or adopt)
        if src is not None and src.model_released and not is_meta_device:
            src.rebuild()
        with HostTimer(sync=False) as t_plan, nvtx_range("reshard/plan"):
            plan = self.plan(src_s, dst_s)
        if self._rank == 0 and os.environ.get("EMB_RESHARD_DEBUG", "0") != "0":
            # per-parameter send / receive plan (the reference's debug print, transfer/transfer.py:271-289)
            print(plan.describe(), flush=True)
        if adopt:
            dst.adopt(src)
            ms, nbytes = 0.0, 0
        elif is_meta_device:
            # meta mode: no data moves; only pre-build state / connections (reference "fake transfer")
            ms, nbytes = 0.0, 0
            if hasattr(self.engine, "warmup"):
                with nvtx_range("reshard/warmup"):
                    self.engine.warmup(plan, self._rank, src, dst, ugroup)
        else:
            with nvtx_range("reshard/transfer"):
                ms, nbytes = self._transfer(plan, src, dst, ugroup)
        with HostTimer(sync=False) as t_lr, nvtx_range("reshard/lr"):
            self._transfer_lr(src, dst, union)
        with HostTimer(sync=False) as t_rel:
            if src is not None and src is not dst and not is_meta_device:
                with nvtx_range("reshard/release"):
                    src.release()
        self.current = dst_s
        set_world_group(ProcessGroupPool.get(dst_s.ranks))
        if dst is not None and not is_meta_device:
            dst.ddp.zero_grad()
            if dst.pool.guard:
                from .memory import check_guards

                check_guards(f"reshard {src_s} -> {dst_s}")
        t_total.__exit__(None, None, None)
        # every phase's time is the MAX over the union ranks (the transfer's is device time)
        mx = max_over_ranks([ms, nbytes / 1e9, t_build.elapsed, t_plan.elapsed, t_lr.elapsed, t_rel.elapsed,
                             t_total.elapsed], group=ProcessGroupPool.get(union, "gloo")
                            if dist.is_initialized() else None)
        el_param = torch.finfo(get_args().model.torch_dtype).bits // 8
        roof = plan.nvlink_roofline_ms(NVLINK_NOMINAL_GBS, 4, el_param)
        meas = measured_link_gbs()
        roof_m = plan.nvlink_roofline_ms(meas, 4, el_param) if meas else None
        links = plan.bytes_matrix(4, el_param)
        np.fill_diagonal(links, 0)
        self.last_switch = {"src": str(src_s), "dst": str(dst_s), "engine": self.engine_name,
                            "transfer_ms": mx[0], "gbytes": mx[1],
                            "bandwidth_gbs": (mx[1] / (mx[0] / 1e3)) if mx[0] > 0 else None,
                            # roofline: busiest GPU's NVLink bytes per direction at the nominal 900 GB/s, and at
                            # the peer-copy rate measured in this job (utils/links.py) when there is one
                            "nvlink_roofline_ms": roof,
                            "roofline_frac": (roof / mx[0]) if mx[0] > 0 else None,
                            "measured_link_gbs": meas,
                            "nvlink_roofline_ms_measured": roof_m,
                            "roofline_frac_measured": (roof_m / mx[0]) if (roof_m is not None and mx[0] > 0) else None,
                            "build_ms": mx[2], "plan_ms": mx[3], "lr_ms": mx[4], "release_ms": mx[5],
                            "total_ms": mx[6],
                            # bytes that cross links, per direction: [sender][receiver] in GB, and the busiest GPU
                            "link_gb": (links / 1e9).round(4).tolist(),
                            "max_egress_gb": float(links.sum(1).max(initial=0)) / 1e9,
                            "max_ingress_gb": float(links.sum(0).max(initial=0)) / 1e9}
        if self._rank == 0 or logger is not None:
            log_json("reshard", logger, **self.last_switch)
        if save_ckpt and dst is not None:
            from .checkpoint import save_checkpoint

            save_checkpoint(dst, os.path.join(ckpt_dir or ".", "after_reshard"))
        return dst

    def recover(self, new_parallel_strategy, failed_ranks, logger: Optional[logging.Logger] = None):
        """Continue on ``new_parallel_strategy`` after ``failed_ranks`` died (detected by ``runtime/health.py``).

        Only the destination ranks take part: they must all be alive, every collective runs on the
        destination's own groups (a dead rank is never waited on), and the plan reads only destination ranks
        that hold source state - typically the surviving Group-ZeRO replica.  Raises ``RuntimeError`` when some
        state has no surviving holder.  Survivors outside the destination just stop (returns ``None``).
        """
        dst_s = ParallelStrategy.from_any(new_parallel_strategy)
        failed = set(failed_ranks)
        assert not (failed & set(dst_s.ranks)), "the recovery strategy must not contain failed ranks"
        src_s = self.current
        if self._rank not in dst_s.ranks:
            self.current = dst_s
            return None
        src = self._states.get(src_s)
        dst = self._get_or_build(dst_s, False)
        plan = build_plan(src_s, dst_s, allowed_src=set(dst_s.ranks) - failed)
        group = ProcessGroupPool.get(dst_s.ranks)
        eng = self.engine
        eng.execute(plan, self._rank, src.param_flat if src else None, src.opt_flat if src else None,
                    dst.param_flat, dst.opt_flat, group)
        if not getattr(eng, "moves_params", True):
            dst.update_model_weight()
        obj = [None]
        if self._rank == 0 and src is not None:
            obj = [{"opt": src.optimizer.state_dict(), "sched": src.opt_param_scheduler.state_dict()}]
        if dist.is_initialized() and dst_s.world_size > 1:
            dist.broadcast_object_list(obj, src=0, group=ProcessGroupPool.get(dst_s.ranks, "gloo"))
        if obj[0] is not None:
            dst.optimizer.load_state_dict(obj[0]["opt"])
            dst.opt_param_scheduler.load_state_dict(obj[0]["sched"])
        if src is not None and src is not dst:
            src.release()
        self.current = dst_s
        set_world_group(ProcessGroupPool.get(dst_s.ranks))
        dst.ddp.zero_grad()
        if self._rank == 0 or logger is not None:
            log_json("recover", logger, src=str(src_s), dst=str(dst_s), failed=sorted(failed))
        return dst

    # ------------------------------------------------------------------ the reference's step-level API
    # The reference's manager exposes the steps of a switch as methods taking its per-strategy state objects
    # (elastic_manager.py:106-178); these take TrainingState objects (or None on ranks outside a strategy) and
    # are what ``reshard`` runs.

    def transfer_params(self, src_state: Optional[TrainingState], dst_state: Optional[TrainingState],
                        union_world_group=None, is_meta_device: bool = False, src_strategy=None,
                        dst_strategy=None) -> float:
        """Move parameters and optimizer state from ``src_state``'s layout to ``dst_state``'s; returns the
        device time in ms (0 in meta mode - or inside ``build_nccl_connection_context`` - which only maps peers
        and builds the task tables).  A rank without state under a layout passes None and names the layout."""
        src_s = self._strategy_of(src_state, src_strategy)
        dst_s = self._strategy_of(dst_state, dst_strategy)
        plan = self.plan(src_s, dst_s)
        ugroup = union_world_group or ProcessGroupPool.get(union_ranks(src_s, dst_s))
        if is_meta_device or self._warm_only:
            if hasattr(self.engine, "warmup"):
                self.engine.warmup(plan, self._rank, src_state, dst_state, ugroup)
            return 0.0
        ms, _ = self._transfer(plan, src_state, dst_state, ugroup)
        return ms

    def redundant_backup(self, src_state: Optional[TrainingState], dst_state: Optional[TrainingState],
                         is_scale_up: bool = False, is_meta_device: bool = False, src_strategy=None,
                         dst_strategy=None) -> float:
        """Group-ZeRO instance-count change.  Dropping replicas (scale-down) and rebuilding them (scale-up) are
        plans like any other switch here, so this is ``transfer_params``; ``is_scale_up`` is accepted for the
        reference's signature."""
        return self.transfer_params(src_state, dst_state, None, is_meta_device, src_strategy, dst_strategy)

    def transfer_learning_rate(self, src_state: Optional[TrainingState], dst_state: Optional[TrainingState],
                               src_strategy=None, dst_strategy=None) -> None:
        """Optimizer step counters, LR and scheduler position from rank 0 to every rank of ``dst_state``."""
        self._transfer_lr(src_state, dst_state, union_ranks(self._strategy_of(src_state, src_strategy),
                                                            self._strategy_of(dst_state, dst_strategy)))

    def log_communication_info(self, transfer_time: float, union_world_group=None,
                               logger: Optional[logging.Logger] = None, nbytes: int = 0) -> Dict:
        """MAX over the union of (transfer ms, GB moved); logged as one JSON line on rank 0 (or to ``logger``).
        ``union_world_group`` must be a host (gloo) group when given."""
        grp = union_world_group
        if grp is None and dist.is_initialized():
            grp = ProcessGroupPool.gloo_world()
        mx = max_over_ranks([transfer_time, nbytes / 1e9], group=grp)
        info = {"transfer_ms": mx[0], "gbytes": mx[1],
                "bandwidth_gbs": (mx[1] / (mx[0] / 1e3)) if mx[0] > 0 else None}
        if self._rank == 0 or logger is not None:
            log_json("communication", logger, **info)
        return info

    @staticmethod
    def _strategy_of(state: Optional[TrainingState], strategy=None) -> ParallelStrategy:
        if state is not None:
            return state.strategy
        if strategy is None:
            raise ValueError("a rank without state under a layout must name the layout (src_strategy / dst_strategy)")
        return ParallelStrategy.from_any(strategy)

    # ------------------------------------------------------------------ internals
    def _transfer(self, plan, src, dst, ugroup):
        eng = self.engine
        if hasattr(eng, "reset_counters"):
            eng.reset_counters()
        sp = src.param_flat if src is not None else None
        so = src.opt_flat if src is not None else None
        dp = dst.param_flat if dst is not None else None
        do = dst.opt_flat if dst is not None else None
        timer = DeviceTimer() if torch.cuda.is_available() else HostTimer(sync=False)
        with timer:
            eng.execute(plan, self._rank, sp, so, dp, do, ugroup)
            if not getattr(eng, "moves_params", True) and dst is not None:
                dst.update_model_weight()
        d = plan.desc
        el_p = torch.finfo(get_args().model.torch_dtype).bits // 8
        mine = d[((d["src_rank"] == self._rank) | (d["dst_rank"] == self._rank)) & (d["src_rank"] != d["dst_rank"])]
        nbytes = int(((mine["rows"] * mine["cols"]) * (mine["kind"] == KIND_OPT) * 12).sum()
                     + ((mine["rows"] * mine["cols"]) * (mine["kind"] == KIND_PARAM) * el_p).sum())
        return timer.elapsed, nbytes

    def _transfer_lr(self, src, dst, union):
        """Optimizer step counters, LR and scheduler position from rank 0 (reference: transfer.py:393-433).

        Rank 0 is always in the union: active ranks are the prefix ``0..world_size-1`` of every strategy."""
        obj = [None]
        if self._rank == 0 and src is not None:
            obj = [{"opt": src.optimizer.state_dict(), "sched": src.opt_param_scheduler.state_dict()}]
        if dist.is_initialized():
            dist.broadcast_object_list(obj, src=0, group=ProcessGroupPool.get(union, "gloo"))
        if dst is not None and obj[0] is not None:
            dst.optimizer.load_state_dict(obj[0]["opt"])
            dst.opt_param_scheduler.load_state_dict(obj[0]["sched"])


@contextlib.contextmanager
def build_nccl_connection_context(manager: "ElasticMegatronManager"):
    """Inside the block the manager's transfers (``transfer_params`` / ``redundant_backup``) only pre-build
    what a switch needs - peer mappings and task tables - and move no data: the reference's "fake transfer",
    used to pay the connection set-up outside the timed switch (elastic_manager.py:268-304).  ``reshard`` has
    the same mode as ``reshard(..., is_meta_device=True)``."""
    prev = manager._warm_only
    manager._warm_only = True
    try:
        yield manager
    finally:
        manager._warm_only = prev
