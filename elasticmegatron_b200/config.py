"""Global model / training configuration.

The reference reads every model and training hyper-parameter from Megatron's global argparse namespace
(``megatron.training.get_args``; consumers listed at elastic_megatron/resharding/virtual_param.py:324-375,
elastic_megatron/megatron_manager/parallel_strategy.py:51-77 and :207-221).  This framework has no Megatron,
so the same role is played by :class:`ModelConfig` + :class:`TrainConfig`, held in one process-wide
:class:`Args` object that :func:`set_args` installs and :func:`get_args` returns.  ``ParallelStrategy``
reads ``num_layers`` / ``num_experts`` from it exactly as the reference reads them from Megatron's args.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class ModelConfig:
    """Architecture of a Llama-style GPT (dense or Mixtral-style MoE)."""

    num_layers: int = 4
    hidden_size: int = 512
    num_attention_heads: int = 8
    num_query_groups: Optional[int] = None  # GQA groups (None -> MHA)
    ffn_hidden_size: int = 1376
    vocab_size: int = 32000
    # The padded vocabulary is frozen for the whole job: it must divide by the largest TP size
    # of every declared strategy, so the vocab-parallel split never changes the tensor shape.
    make_vocab_size_divisible_by: int = 128
    max_tensor_parallel_size: int = 8
    seq_length: int = 512
    rotary_base: float = 10000.0
    norm_epsilon: float = 1e-5
    # "RMSNorm" (Llama) or "LayerNorm" (Megatron's default, with a bias per norm: the reference's demo model)
    normalization: str = "RMSNorm"
    init_method_std: float = 0.02
    untie_embeddings_and_output_weights: bool = True
    # MoE
    num_experts: Optional[int] = None
    moe_router_topk: int = 2
    moe_aux_loss_coeff: float = 1e-2
    moe_ffn_hidden_size: Optional[int] = None
    # numerics
    params_dtype: str = "bf16"  # "bf16" | "fp32"

    def __post_init__(self):
        if self.num_query_groups is None:
            self.num_query_groups = self.num_attention_heads
        if self.num_experts == 0:
            self.num_experts = None
        if self.moe_ffn_hidden_size is None:
            self.moe_ffn_hidden_size = self.ffn_hidden_size
        assert self.hidden_size % self.num_attention_heads == 0
        assert self.num_attention_heads % self.num_query_groups == 0
        if self.normalization not in ("RMSNorm", "LayerNorm"):
            raise ValueError(f"normalization must be RMSNorm or LayerNorm, got {self.normalization!r}")

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def heads_per_group(self) -> int:
        return self.num_attention_heads // self.num_query_groups

    @property
    def qkv_rows(self) -> int:
        """Rows of the fused QKV weight: per query group [q heads | k | v] x head_dim."""
        return self.num_query_groups * (self.heads_per_group + 2) * self.head_dim

    @property
    def padded_vocab_size(self) -> int:
        mult = self.make_vocab_size_divisible_by * self.max_tensor_parallel_size
        return int(math.ceil(self.vocab_size / mult) * mult)

    @property
    def is_moe(self) -> bool:
        return bool(self.num_experts)

    @property
    def torch_dtype(self):
        import torch

        return {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}[self.params_dtype]

    def num_params(self) -> int:
        h, f, v = self.hidden_size, self.ffn_hidden_size, self.padded_vocab_size
        norm = 2 * h if self.normalization == "LayerNorm" else h  # weight (+ bias)
        per_layer = self.qkv_rows * h + h * h + 2 * norm
        if self.is_moe:
            per_layer += self.num_experts * (3 * self.moe_ffn_hidden_size * h) + self.num_experts * h
        else:
            per_layer += 3 * f * h
        emb = v * h * (2 if self.untie_embeddings_and_output_weights else 1)
        return self.num_layers * per_layer + emb + norm


@dataclass
class TrainConfig:
    micro_batch_size: int = 1
    global_batch_size: int = 8
    lr: float = 3e-4
    min_lr: float = 3e-5
    lr_warmup_iters: int = 0
    lr_decay_iters: Optional[int] = None
    lr_decay_style: str = "cosine"
    train_iters: int = 100
    weight_decay: float = 0.1
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_eps: float = 1e-8
    clip_grad: float = 1.0
    seed: int = 0
    # DDP / ZeRO
    use_distributed_optimizer: bool = True
    overlap_grad_reduce: bool = False
    # leave the parameter all-gathers after the optimizer step in flight; the next forward waits per bucket
    # (Megatron's --overlap-param-gather)
    overlap_param_gather: bool = False
    ddp_bucket_size: Optional[int] = None
    grad_reduce_in_fp32: bool = True
    # memory: recompute every transformer layer's activations in backward (keep only layer inputs)
    recompute: bool = False
    # context parallelism: "all_gather" (K/V gathered over the CP group), "p2p" (K/V passed round a ring) or
    # "a2a" (Ulysses: all-to-all from a sequence split to a query-group split and back)
    cp_comm_type: str = "all_gather"

    def __post_init__(self):
        # Megatron flags kept for familiarity; the training core implements one setting of each
        if not self.use_distributed_optimizer:
            raise ValueError("the optimizer state is always sharded over the DP*CP ranks (ZeRO-1); for a replicated "
                             "optimizer give the strategy num_distributed_optimizer_instances = DP*CP")
        if not self.grad_reduce_in_fp32:
            raise ValueError("gradients always accumulate and reduce in fp32 (main_grad)")
        if self.lr_decay_style not in ("cosine", "linear", "constant"):
            raise ValueError(f"lr_decay_style must be cosine, linear or constant, got {self.lr_decay_style!r}")
        if self.cp_comm_type not in ("all_gather", "p2p", "a2a"):
            raise ValueError(f"cp_comm_type must be all_gather, p2p or a2a, got {self.cp_comm_type!r}")


@dataclass
class Args:
    """Process-wide configuration (the analogue of Megatron's global ``args``)."""

    model: ModelConfig = field(default_factory=ModelConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    consumed_train_samples: int = 0
    iteration: int = 0

    # Convenience accessors under the names the reference reads from Megatron's args.
    @property
    def num_layers(self):
        return self.model.num_layers

    @property
    def num_experts(self):
        return self.model.num_experts

    @property
    def padded_vocab_size(self):
        return self.model.padded_vocab_size

    @property
    def hidden_size(self):
        return self.model.hidden_size


_ARGS: Optional[Args] = None


def set_args(args: Args) -> Args:
    global _ARGS
    _ARGS = args
    return args


def get_args() -> Args:
    global _ARGS
    if _ARGS is None:
        _ARGS = Args()
    return _ARGS


def replace(obj, **kw):
    return dataclasses.replace(obj, **kw)


# Named architectures used by the benchmarks and tests (shapes from the reference's launch scripts and
# the benchmark configs: run_e2e_demo.sh:77-95, run_moe.sh:38-68).
PRESETS = {
    "tiny-llama": dict(num_layers=4, hidden_size=512, num_attention_heads=8, ffn_hidden_size=1376,
                       vocab_size=32000, seq_length=512, params_dtype="fp32"),
    "llama2-7b": dict(num_layers=32, hidden_size=4096, num_attention_heads=32, ffn_hidden_size=11008,
                      vocab_size=32000, seq_length=4096),
    "llama2-13b": dict(num_layers=40, hidden_size=5120, num_attention_heads=40, ffn_hidden_size=13824,
                       vocab_size=32000, seq_length=4096),
    "llama3-8b": dict(num_layers=32, hidden_size=4096, num_attention_heads=32, num_query_groups=8,
                      ffn_hidden_size=14336, vocab_size=128256, seq_length=8192, rotary_base=500000.0),
    # the reference demo's default model (run_e2e_demo.sh:25-31, MODEL_SIZE=tiny): Megatron's LayerNorm, MHA
    "demo-tiny": dict(num_layers=4, hidden_size=4096, num_attention_heads=32, ffn_hidden_size=11008,
                      vocab_size=32000, seq_length=4096, normalization="LayerNorm"),
    "mixtral-8x7b": dict(num_layers=32, hidden_size=4096, num_attention_heads=32, num_query_groups=8,
                         ffn_hidden_size=14336, vocab_size=32000, seq_length=4096, num_experts=8,
                         moe_router_topk=2, moe_aux_loss_coeff=1e-2, rotary_base=1e6),
}


def preset(name: str, **overrides) -> ModelConfig:
    d = dict(PRESETS[name])
    d.update(overrides)
    return ModelConfig(**d)
