"""``TrainingState``: model + optimizer + scheduler of one strategy, over pooled flat arenas.

Reference counterpart: elastic_megatron/megatron_manager/training_state.py (427 lines) which holds Megatron
model chunks / optimizer / scheduler and frees memory without destroying tensor objects.  Here the stage's
parameters, ``main_grad`` views and the optimizer all point into three arenas (param, grad, optimizer) that
``release_*`` hands back to the pool and ``rebuild_*`` takes again; every Python object (modules, hooks,
optimizer, scheduler) survives a release.
"""
from __future__ import annotations

import contextlib

from typing import Callable, Dict, List, Optional

import torch

from ..config import ModelConfig, TrainConfig, get_args
from ..models.llama import GPTStage
from ..parallel.ddp import DistributedDataParallel
from ..parallel.optimizer import DistributedAdam
from ..parallel.process_groups import ParallelState
from ..parallel.scheduler import OptimizerParamScheduler
from ..parallel.strategy import ParallelStrategy
from ..planner.layout import RankLayout, rank_layout
from .memory import Arena, get_pool


class StepHooks:
    """The per-layout hooks a training loop calls around forward / backward (see ``TrainingState.refresh_config``)."""

    def __init__(self, ddp):
        self.ddp = ddp

    @contextlib.contextmanager
    def no_sync_func(self):
        prev = self.ddp.sync_enabled
        self.ddp.sync_enabled = False
        try:
            yield
        finally:
            self.ddp.sync_enabled = prev

    def grad_sync_func(self) -> None:
        self.ddp.finish_grad_sync()

    def param_sync_func(self, overlap: bool = False) -> None:
        self.ddp.start_param_sync(overlap=overlap)

    @staticmethod
    def grad_scale_func(loss):
        return loss


class TrainingState:
    setup_model_and_optimizer_func: Optional[Callable] = None

    @classmethod
    def set_setup_model_and_optimizer_func(cls, fn: Callable) -> None:
        assert callable(fn)
        cls.setup_model_and_optimizer_func = fn

    def __init__(self, strategy: ParallelStrategy, cfg: Optional[ModelConfig] = None,
                 train_cfg: Optional[TrainConfig] = None, device=None, is_meta_device: bool = False):
        args = get_args()
        from .meta import in_meta_context

        is_meta_device = is_meta_device or in_meta_context()
        self.cfg = cfg or args.model
        self.train_cfg = train_cfg or args.train
        self.strategy = strategy
        self.ps = ParallelState(strategy)
        self.rank = self.ps.rank
        self.is_meta_device = is_meta_device
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else \
                torch.device("cpu")
        self.device = torch.device(device)
        self.pool = get_pool(self.device)
        tc = self.train_cfg
        self.layout: RankLayout = rank_layout(self.cfg, strategy, self.rank, tc.overlap_grad_reduce,
                                              tc.ddp_bucket_size)
        self.param_dtype = self.cfg.torch_dtype
        if self.device.type == "cuda" and not is_meta_device and self.param_dtype != torch.bfloat16:
            raise ValueError(f"CUDA training runs in bf16 (params_dtype={self.cfg.params_dtype}); fp32 parameters "
                             "are the CPU (gloo) path")
        self.param_arena: Optional[Arena] = None
        self.grad_arena: Optional[Arena] = None
        self.opt_arena: Optional[Arena] = None
        if not is_meta_device:
            self._alloc_model()
            self._alloc_opt()
        views = self._param_views() if not is_meta_device else self._meta_views()
        self.stage = GPTStage(self.cfg, self.ps, self.layout.params, views, tc.micro_batch_size, tc.cp_comm_type,
                              tc.recompute)
        self.stage._training_state = self
        self.model = [self.stage]
        self.ddp = DistributedDataParallel(self.layout, self.ps, self.stage.params_by_name, self.param_flat,
                                           self.grad_flat, tc.overlap_grad_reduce)
        self.optimizer = DistributedAdam(self.layout, self.ps, self.param_flat, self.grad_flat, self.opt_flat, tc)
        gbs = tc.global_batch_size
        decay = (tc.lr_decay_iters or tc.train_iters) * gbs
        self.opt_param_scheduler = OptimizerParamScheduler(self.optimizer, tc.lr, tc.min_lr,
                                                           tc.lr_warmup_iters * gbs, decay, tc.lr_decay_style)
        self.model_released = is_meta_device
        self.optimizer_released = is_meta_device

    # ------------------------------------------------------------------ arenas
    @property
    def param_flat(self) -> Optional[torch.Tensor]:
        # a reader of the whole arena (switch, checkpoint, checksum) must see the gathered parameters: wait for
        # any all-gather the last step left in flight (no-op otherwise)
        ddp = self.__dict__.get("ddp")
        if ddp is not None:
            ddp.wait_params()
        return self.param_arena.view(self.param_dtype, (self.layout.param_numel,)) if self.param_arena else None

    @property
    def grad_flat(self) -> Optional[torch.Tensor]:
        return self.grad_arena.view(torch.float32, (self.layout.param_numel,)) if self.grad_arena else None

    @property
    def opt_flat(self) -> Optional[torch.Tensor]:
        return self.opt_arena.view(torch.float32, (3, self.layout.opt_numel)) if self.opt_arena else None

    def _alloc_model(self):
        n = self.layout.param_numel
        el = torch.finfo(self.param_dtype).bits // 8
        self.param_arena = self.pool.alloc(n * el)
        self.grad_arena = self.pool.alloc(n * 4)
        # padding elements must be zero (they travel in all-gathers and reductions)
        self.param_flat.zero_()
        self.grad_flat.zero_()

    def _alloc_opt(self):
        self.opt_arena = self.pool.alloc(3 * self.layout.opt_numel * 4)
        self.opt_flat.zero_()

    def _param_views(self) -> Dict[str, torch.Tensor]:
        P = self.param_flat
        return {lp.name: P[self.layout.offset_by_name[lp.name]:self.layout.offset_by_name[lp.name] + lp.numel]
                .view(lp.shape) for lp in self.layout.params}

    def _meta_views(self) -> Dict[str, torch.Tensor]:
        return {lp.name: torch.empty(lp.shape, dtype=self.param_dtype, device="meta") for lp in self.layout.params}

    def release_model(self) -> None:
        if self.model_released:
            return
        if self.__dict__.get("ddp") is not None:
            self.ddp.wait_params()  # no all-gather may still write into the arena handed back to the pool
        self.pool.free(self.param_arena)
        self.pool.free(self.grad_arena)
        self.param_arena = self.grad_arena = None
        self.model_released = True

    def release_optimizer(self) -> None:
        if self.optimizer_released:
            return
        self.pool.free(self.opt_arena)
        self.opt_arena = None
        self.optimizer_released = True

    def rebuild_model(self) -> None:
        if not self.model_released:
            return
        self._alloc_model()
        self._bind_model_arenas()

    def _bind_model_arenas(self) -> None:
        """Point the model, DDP and optimizer at the current param / grad arenas."""
        if self.is_meta_device:
            # meta parameters cannot be re-pointed at device memory in place: build the stage and its
            # gradient hooks afresh over the new arenas (the optimizer and scheduler objects survive)
            self.ddp.remove_hooks()
            self.stage = GPTStage(self.cfg, self.ps, self.layout.params, self._param_views(),
                                  self.train_cfg.micro_batch_size, self.train_cfg.cp_comm_type,
                                  self.train_cfg.recompute)
            self.stage._training_state = self
            self.model = [self.stage]
            self.ddp = DistributedDataParallel(self.layout, self.ps, self.stage.params_by_name, self.param_flat,
                                               self.grad_flat, self.train_cfg.overlap_grad_reduce)
        else:
            self.stage.rebind(self._param_views())
        self.ddp.bind(self.param_flat, self.grad_flat)
        self.optimizer.bind(self.param_flat, self.grad_flat, self.opt_flat)
        self.model_released = False
        self.is_meta_device = False

    def rebuild_optimizer(self) -> None:
        if not self.optimizer_released:
            return
        self._alloc_opt()
        self.optimizer.bind(self.param_flat, self.grad_flat, self.opt_flat)
        self.optimizer_released = False

    def release(self):
        self.release_model()
        self.release_optimizer()

    def adopt(self, other: "TrainingState") -> None:
        """Take over ``other``'s arenas instead of copying them; ``other`` ends released.

        Valid when both layouts are the same (strategies that differ only in sequence parallelism: the layout
        does not depend on it), so every parameter, gradient and optimizer element already sits at its offset
        under this strategy."""
        lo, ls = other.layout, self.layout
        assert (lo.offset_by_name == ls.offset_by_name and lo.param_numel == ls.param_numel
                and lo.owned() == ls.owned()), "adopt needs identical layouts"
        self.release()
        self.param_arena, self.grad_arena, self.opt_arena = other.param_arena, other.grad_arena, other.opt_arena
        other.param_arena = other.grad_arena = other.opt_arena = None
        other.model_released = other.optimizer_released = True
        self._bind_model_arenas()
        self.optimizer.bind(self.param_flat, self.grad_flat, self.opt_flat)
        self.optimizer_released = False

    def rebuild(self):
        self.rebuild_model()
        self.rebuild_optimizer()

    # ------------------------------------------------------------------ init
    def init_weights(self, seed: int = 0, method: str = "global") -> None:
        """Random-init params (N(0, std), norms = 1) and set master = param, moments = 0.

        ``global``: layout-independent values (every strategy holds the same model; small models / tests).
        ``local``: device-side per-shard init, identical across DP replicas (fast; benchmarks).
        """
        P, O = self.param_flat, self.opt_flat
        P.zero_()
        O.zero_()
        if method == "global":
            from ..planner.materialize import init_global_params, scatter_to_rank

            g = init_global_params(self.cfg, seed)
            g = {k: v.to(self.param_dtype).float() for k, v in g.items()}
            Pc = torch.zeros(P.shape, dtype=torch.float32)
            Oc = torch.zeros(O.shape, dtype=torch.float32)
            scatter_to_rank(self.cfg, self.strategy, self.rank, g, Pc, Oc, None, self.train_cfg.overlap_grad_reduce,
                            self.train_cfg.ddp_bucket_size)
            P.copy_(Pc.to(self.param_dtype))
            O.copy_(Oc)
        else:
            c = self.strategy.coords(self.rank)
            for lp in self.layout.params:
                off = self.layout.offset_by_name[lp.name]
                vp = lp.members[0][0]
                v = P[off:off + lp.numel]
                if vp.init == "ones":
                    v.fill_(1.0)
                elif vp.init == "zeros":
                    v.zero_()
                else:
                    gen = torch.Generator(device=P.device)
                    gen.manual_seed(seed * 7919 + vp.index * 131 + (c["etp"] if lp.is_expert else c["tp"]) * 17
                                    + (c["ep"] if lp.is_expert else 0))
                    v.normal_(0.0, self.cfg.init_method_std, generator=gen)
            for a, o, n, wd, cnt in self.optimizer.segs:
                O[0, o:o + n].copy_(P[a:a + n].float())

    # ------------------------------------------------------------------ misc (reference API)
    @property
    def optimizers(self):
        return [self.optimizer]

    @staticmethod
    def refresh_config(model, optimizer):
        """Bind the step hooks of the layout that owns ``model`` (reference: training_state.py:110-135, which
        points Megatron's model config at the new DDP's ``no_sync`` / ``start_grad_sync`` / ``start_param_sync``
        and the optimizer's loss scaling after a switch).

        Returns a :class:`StepHooks` and stores it on every model chunk as ``step_hooks``: ``no_sync_func`` (a
        context in which backward only accumulates gradients), ``grad_sync_func`` (finish the DP reduction of
        the step), ``param_sync_func`` (start the parameter all-gathers, in flight until the forward needs each
        bucket when ``overlap`` is true) and ``grad_scale_func`` (bf16 training has no loss scale: identity).
        Custom training loops call these instead of holding on to a previous layout's DDP."""
        chunks = list(model) if isinstance(model, (list, tuple)) else [model]
        ts = chunks[0].__dict__.get("_training_state") if chunks else None
        if ts is None:
            raise ValueError("refresh_config: the model does not belong to a TrainingState")
        if optimizer is not None and optimizer is not ts.optimizer:
            raise ValueError("refresh_config: the optimizer belongs to another layout than the model")
        hooks = StepHooks(ts.ddp)
        for c in chunks:
            c.step_hooks = hooks
        return hooks

    def update_model_weight(self) -> None:
        """Regenerate params from the fp32 master of the own shard and all-gather over DP (reference:
        training_state.py:176-197).  The direct transfer engine already delivers params, so the manager only
        calls this for engines that move optimizer state alone."""
        P, O = self.param_flat, self.opt_flat
        for a, o, n, wd, c in self.optimizer.segs:
            P[a:a + n].copy_(O[0, o:o + n].to(P.dtype))
        self.ddp.start_param_sync()

    def save_checkpoint(self, path: str, iteration: Optional[int] = None) -> str:
        """Megatron legacy checkpoint of this layout (collective over the strategy's ranks; reference:
        training_state.py:325-366)."""
        from .checkpoint import save_checkpoint

        return save_checkpoint(self, path, iteration)

    def get_metadata(self) -> Dict:
        """Where this rank's state lives: strategy, arena sizes and the ZeRO segments of the optimizer (the
        reference keeps per-parameter metadata for its planner, training_state.py:145-174; here the layout is a
        pure function of the strategy, so this is a description, not an input)."""
        return {"strategy": self.strategy.to_dict(), "rank": self.rank,
                "param_numel": self.layout.param_numel, "opt_numel": self.layout.opt_numel,
                "segments": [(int(a), int(o), int(n)) for a, o, n, *_ in self.optimizer.segs],
                "model_released": self.model_released, "optimizer_released": self.optimizer_released}

    def all_optimizer_tensors(self) -> List[torch.Tensor]:
        """fp32 master, exp_avg and exp_avg_sq of this rank's shard (views into the optimizer arena)."""
        O = self.opt_flat
        return [] if O is None else [O[0], O[1], O[2]]
