"""Learning-rate schedule: linear warm-up then cosine / linear / constant decay to ``min_lr``, counted in samples.

Same contract as the Megatron ``OptimizerParamScheduler`` the reference carries across switches
(elastic_megatron/megatron_manager/training_state.py:369-427; transfer.py:393-433): ``step(increment)``
advances by ``num_microbatches * micro_batch_size * DP`` samples, and ``state_dict`` / ``load_state_dict``
restore the position without stepping.
"""
from __future__ import annotations

import math
from typing import Dict


class OptimizerParamScheduler:
    def __init__(self, optimizer, max_lr: float, min_lr: float, lr_warmup_steps: int, lr_decay_steps: int,
                 lr_decay_style: str = "cosine", init_lr: float = 0.0):
        self.optimizer = optimizer
        self.max_lr, self.min_lr, self.init_lr = float(max_lr), float(min_lr), float(init_lr)
        self.lr_warmup_steps = int(lr_warmup_steps)
        self.lr_decay_steps = max(int(lr_decay_steps), 1)
        self.lr_decay_style = lr_decay_style
        self.num_steps = 0
        self.step(0)

    def get_lr(self) -> float:
        n = self.num_steps
        if self.lr_warmup_steps > 0 and n <= self.lr_warmup_steps:
            return self.init_lr + (self.max_lr - self.init_lr) * n / self.lr_warmup_steps
        if self.lr_decay_style == "constant":
            return self.max_lr
        if n > self.lr_decay_steps:
            return self.min_lr
        span = self.lr_decay_steps - self.lr_warmup_steps
        ratio = (n - self.lr_warmup_steps) / span if span > 0 else 1.0
        if self.lr_decay_style == "linear":
            coeff = 1.0 - ratio
        elif self.lr_decay_style == "cosine":
            coeff = 0.5 * (math.cos(math.pi * ratio) + 1.0)
        else:
            raise ValueError(self.lr_decay_style)
        return self.min_lr + coeff * (self.max_lr - self.min_lr)

    def step(self, increment: int) -> None:
        self.num_steps += increment
        lr = self.get_lr()
        for g in getattr(self.optimizer, "param_groups", []):
            g["lr"] = lr

    def state_dict(self) -> Dict:
        return {"max_lr": self.max_lr, "min_lr": self.min_lr, "init_lr": self.init_lr,
                "lr_warmup_steps": self.lr_warmup_steps, "lr_decay_steps": self.lr_decay_steps,
                "lr_decay_style": self.lr_decay_style, "num_steps": self.num_steps}

    def load_state_dict(self, sd: Dict) -> None:
        """Restore without stepping (reference: load_state_dict_with_no_step, training_state.py:369-378)."""
        for k in ("max_lr", "min_lr", "init_lr", "lr_warmup_steps", "lr_decay_steps", "lr_decay_style",
                  "num_steps"):
            if k in sd:
                setattr(self, k, sd[k])
        lr = self.get_lr()
        for g in getattr(self.optimizer, "param_groups", []):
            g["lr"] = lr
