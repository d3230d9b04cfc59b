"""Llama-style GPT (dense SwiGLU or Mixtral-style MoE) as one pipeline stage.

Activations are 2-D ``[tokens, features]`` with the sequence as the outer index (token = s * b + b_idx), so
sequence parallelism and context parallelism split dim 0 contiguously.  Parameters are plain views into the
rank's flat parameter arena (``runtime/training_state.py``); the stage never allocates its own weights, which
is what lets a reshard swap the arena underneath it.

Parallel structure per layer (Megatron-style, behaviour inferred from the reference's launch flags,
run_e2e_demo.sh:77-95 and run_moe.sh:38-68):

* input RMSNorm -> column-parallel QKV (AG over SP) -> RoPE -> causal GQA attention (ring over CP) ->
  row-parallel proj (RS over SP) -> residual;
* RMSNorm -> column-parallel fc1 ``[W_t; V_t]`` -> SwiGLU -> row-parallel fc2 -> residual; or for MoE:
  router (softmax over the top-k logits, switch load-balancing aux loss) -> all-to-all dispatch over EP ->
  grouped expert SwiGLU MLPs -> all-to-all combine.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.utils.checkpoint
from torch import nn

from ..config import ModelConfig
from ..ops import functional as F_
from ..ops import reference as ref
from ..models.spec import LocalParam
from .moe import MoELayer
from ..parallel.context_parallel import CP_COMM_TYPES, cp_attention, cp_ring_attention, cp_ulysses_attention


class RotaryCache:
    def __init__(self):
        self._c: Dict[tuple, tuple] = {}

    def get(self, positions: torch.Tensor, dim: int, base: float, device):
        key = (positions.shape[0], int(positions[0]), int(positions[-1]), dim, base, str(device))
        v = self._c.get(key)
        if v is None:
            cos, sin = ref.rope_cos_sin(positions.cpu(), dim, base)
            v = (cos.to(device), sin.to(device))
            self._c[key] = v
        return v


_ROPE = RotaryCache()


def cp_positions(seq: int, cp: int, cp_rank: int) -> torch.Tensor:
    """Global positions of the tokens a CP rank holds: chunks (r, 2cp-1-r) of 2cp equal chunks."""
    if cp == 1:
        return torch.arange(seq)
    c = seq // (2 * cp)
    a = torch.arange(cp_rank * c, (cp_rank + 1) * c)
    b = torch.arange((2 * cp - 1 - cp_rank) * c, (2 * cp - cp_rank) * c)
    return torch.cat([a, b])


class GPTStage(nn.Module):
    def __init__(self, cfg: ModelConfig, pstate, params: List[LocalParam], views: Dict[str, torch.Tensor],
                 micro_batch_size: int, cp_comm_type: str = "all_gather", recompute: bool = False):
        super().__init__()
        if cp_comm_type not in CP_COMM_TYPES:
            raise ValueError(f"cp_comm_type must be one of {CP_COMM_TYPES}, got {cp_comm_type!r}")
        self.cfg, self.ps = cfg, pstate
        s = pstate.strategy
        self.tp = s.tensor_model_parallel_size
        self.sp = bool(s.sequence_parallel) and self.tp > 1
        self.cp = s.context_parallel_size
        self.first, self.last = pstate.is_first_stage, pstate.is_last_stage
        self.mbs = micro_batch_size
        # full activation recompute, one transformer layer per checkpoint (Megatron's --recompute-granularity
        # full --recompute-method uniform --recompute-num-layers 1, which the reference's MoE launcher uses,
        # run_moe.sh:101-105): only each layer's input is kept; backward replays the layer's forward
        self.recompute = recompute
        self.tp_group = pstate.group("tp") if self.tp > 1 else None
        self.cp_group = pstate.group("cp") if self.cp > 1 else None
        self.cp_attention = {"all_gather": cp_attention, "p2p": cp_ring_attention,
                             "a2a": cp_ulysses_attention}[cp_comm_type]
        if self.cp > 1 and cp_comm_type == "a2a" and (cfg.num_query_groups // self.tp) % self.cp:
            raise ValueError(f"cp_comm_type a2a needs the query groups per TP rank "
                             f"({cfg.num_query_groups // self.tp}) divisible by CP ({self.cp})")
        self.params_by_name: Dict[str, nn.Parameter] = {}
        for lp in params:
            p = nn.Parameter(views[lp.name], requires_grad=True)
            p._local_param = lp
            self.params_by_name[lp.name] = p
        # register under sanitized names so .parameters() / state_dict work
        for n, p in self.params_by_name.items():
            self.register_parameter(n.replace(".", "__"), p)
        self.num_local_layers = len({lp.layer_local for lp in params if lp.layer_local is not None})
        self.moe = [MoELayer(cfg, pstate, self._p(i, "mlp.router.weight"), self._p(i, "mlp.experts.linear_fc1.weight"),
                             self._p(i, "mlp.experts.linear_fc2.weight"))
                    for i in range(self.num_local_layers)] if cfg.is_moe else None
        self.vocab_start = pstate.tp_rank * (cfg.padded_vocab_size // self.tp) if self.tp > 1 else 0

    def _p(self, layer: int, key: str) -> nn.Parameter:
        return self.params_by_name[f"decoder.layers.{layer}.{key}"]

    def _norm(self, x: torch.Tensor, weight_name: str) -> torch.Tensor:
        """RMSNorm (native kernel), or LayerNorm with the bias stored next to the weight."""
        w = self.params_by_name[weight_name]
        if self.cfg.normalization == "LayerNorm":
            b = self.params_by_name[weight_name[:-len("weight")] + "bias"]
            return F_.layernorm(x, w, b, self.cfg.norm_epsilon)
        return F_.rmsnorm(x, w, self.cfg.norm_epsilon)

    def _add_norm(self, x: torch.Tensor, pending: Optional[torch.Tensor], weight_name: str):
        """Residual add of the previous branch's output (``pending``) fused into the norm that follows it:
        returns (the new residual stream, its normalised copy)."""
        if pending is None:
            return x, self._norm(x, weight_name)
        if self.cfg.normalization == "LayerNorm":
            x = x + pending
            return x, self._norm(x, weight_name)
        return F_.add_rmsnorm(x, pending, self.params_by_name[weight_name], self.cfg.norm_epsilon)

    def _wait_params(self, key) -> None:
        """Wait for the parameter all-gathers (left in flight by the last optimizer step) of the buckets that
        hold the parameters read first by ``key`` (local layer index, 'pre', 'post')."""
        ts = self.__dict__.get("_training_state")
        ddp = ts.__dict__.get("ddp") if ts is not None else None
        if ddp is not None:
            ddp.wait_params(key)

    def rebind(self, views: Dict[str, torch.Tensor]) -> None:
        """Point every parameter at a new arena (after a release / rebuild)."""
        for n, p in self.params_by_name.items():
            p.data = views[n]

    # ------------------------------------------------------------------------------------------ forward
    def _mode(self, kind: str) -> Optional[str]:
        if self.tp == 1:
            return None
        return f"{kind}_sp" if self.sp else kind

    def forward(self, inp: torch.Tensor, labels: Optional[torch.Tensor] = None):
        cfg = self.cfg
        seq_local = cfg.seq_length // self.cp
        b = self.mbs
        self._wait_params("pre")
        if self.first:
            # inp: token ids [b, s_local] -> [s_local * b] seq-major
            ids = inp.t().contiguous().view(-1)
            x = F_.embedding(ids, self.params_by_name["embedding.word_embeddings.weight"], self.vocab_start)
            if self.tp > 1:
                x = F_.reduce_scatter_to_sp(x, self.tp_group) if self.sp else F_.reduce_from_tp(x, self.tp_group)
        else:
            x = inp
        positions = cp_positions(cfg.seq_length, self.cp, self.ps.cp_rank if self.cp > 1 else 0)
        cos, sin = _ROPE.get(positions, cfg.head_dim, cfg.rotary_base, x.device)
        aux_total = None
        recompute = self.recompute and torch.is_grad_enabled()
        # the residual stream is carried as (x, pending): the last branch output is added by the norm that
        # consumes it (the next layer's input norm, or the final norm)
        pending = None
        for i in range(self.num_local_layers):
            self._wait_params(i)
            if recompute:
                # early stop off: every rank replays the whole layer, so its collectives run in full and in
                # the same order on all ranks of each group
                with torch.utils.checkpoint.set_checkpoint_early_stop(False):
                    x, pending, aux = torch.utils.checkpoint.checkpoint(self._layer, i, x, pending, cos, sin,
                                                                        seq_local, b, use_reentrant=False)
            else:
                x, pending, aux = self._layer(i, x, pending, cos, sin, seq_local, b)
            if aux is not None:
                aux_total = aux if aux_total is None else aux_total + aux
        if not self.last:
            return (x + pending if pending is not None else x), aux_total
        self._wait_params("post")
        _, x = self._add_norm(x, pending, "decoder.final_layernorm.weight")
        # untied, or the last stage's copy of a tied embedding; at PP=1 a tied head is the embedding itself
        w_out = self.params_by_name.get("output_layer.weight")
        if w_out is None:
            w_out = self.params_by_name["embedding.word_embeddings.weight"]
        logits = F_.linear(x, w_out, self._mode("col"), self.tp_group)
        lab = labels.t().contiguous().view(-1)
        losses = F_.vocab_parallel_cross_entropy(logits, lab, self.vocab_start, self.tp_group)
        return losses, aux_total

    def _layer(self, i: int, x: torch.Tensor, pending: Optional[torch.Tensor], cos, sin, seq_local: int, b: int):
        """One transformer layer on the residual stream ``x + pending``; returns (x', pending', aux) with the
        layer's output equal to ``x' + pending'`` (the MLP branch's output is left for the next norm to add)."""
        cfg = self.cfg
        G_loc = cfg.num_query_groups // self.tp
        hpg, d = cfg.heads_per_group, cfg.head_dim
        x, h = self._add_norm(x, pending, f"decoder.layers.{i}.self_attention.linear_qkv.layer_norm_weight")
        qkv = F_.linear(h, self._p(i, "self_attention.linear_qkv.weight"), self._mode("col"), self.tp_group)
        qkv = qkv.view(seq_local, b, G_loc, hpg + 2, d)
        qkv = F_.rope_qkv(qkv, cos, sin, hpg + 1)
        if self.cp > 1:
            attn = self.cp_attention(qkv, hpg, self.cp_group, self.ps.cp_rank, self.cp)
        else:
            attn = F_.attention(qkv, hpg)
        o = F_.linear(attn.view(seq_local * b, -1), self._p(i, "self_attention.linear_proj.weight"),
                      self._mode("row"), self.tp_group)
        aux = None
        if self.moe is not None:
            x, h = self._add_norm(x, o, f"decoder.layers.{i}.pre_mlp_layernorm.weight")
            o, aux = self.moe[i](h)
        else:
            x, h = self._add_norm(x, o, f"decoder.layers.{i}.mlp.linear_fc1.layer_norm_weight")
            h = F_.linear(h, self._p(i, "mlp.linear_fc1.weight"), self._mode("col"), self.tp_group)
            h = F_.swiglu(h)
            o = F_.linear(h, self._p(i, "mlp.linear_fc2.weight"), self._mode("row"), self.tp_group)
        return x, o, aux
