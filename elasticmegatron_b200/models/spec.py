"""Layout-independent description of a model's parameters (the "virtual parameter space").

The reference reconstructs this description from the first local layer of a live Megatron model and
replicates it ``num_layers`` times (elastic_megatron/resharding/virtual_param.py:472-802), classifying each
parameter by name regex (elastic_megatron/resharding/resharding_metadata.py:322-386).  Here the model is our
own, so the description is generated directly from :class:`ModelConfig`, and the runtime model, the DDP
buffer layout, the checkpoint writer and the reshard planner all read it from this one module.

Global (TP=PP=EP=1) layout conventions, which fix what a TP/EP split means:

* ``linear_qkv.weight`` ``[G*(H/G+2)*d, h]``: rows grouped per query group ``g`` as
  ``[q heads of g | k_g | v_g]``, so a contiguous dim-0 split is a set of whole groups (GQA-safe);
* ``linear_fc1.weight`` ``[2f, h]`` = ``[W; V]`` (gate; up).  TP rank ``t`` of ``T`` holds ``[W_t; V_t]``,
  i.e. two row blocks - the reference performs this permutation with explicit shuffle copies
  (resharding_metadata.py:98-178); here it is an index map (``tp_kind="swiglu"``);
* row-parallel weights (``linear_proj``, ``linear_fc2``) split dim 1;
* vocab-parallel ``word_embeddings`` / ``output_layer`` split dim 0 of the *padded* vocab, which is frozen
  for the job (it divides by the largest TP of every strategy);
* each expert is its own virtual parameter; on an EP rank the local experts are stacked in one tensor
  ``[E_local, ...]`` (grouped-GEMM order) and a virtual expert maps to one slice of it.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from ..config import ModelConfig

PRE, LAYER, POST = "pre", "layer", "post"


@dataclass(frozen=True)
class VParam:
    """One virtual parameter in its global (unsharded) form."""

    index: int
    name: str  # global name with the global layer index / global expert id
    shape: Tuple[int, ...]
    tp_dim: Optional[int] = None  # None -> replicated across TP
    tp_kind: str = "plain"  # "plain" | "swiglu"
    stage_kind: str = LAYER
    layer_id: Optional[int] = None
    expert_id: Optional[int] = None
    sp_partial: bool = False  # grad is a partial sum across TP ranks under sequence parallelism
    weight_decay: bool = True
    init: str = "normal"  # "normal" | "ones" | "zeros"
    # name of the model parameter (within a layer / stage) this virtual param lives in
    local_key: str = ""
    # the word embedding also serves as the output layer (untie_embeddings_and_output_weights=False)
    tied_head: bool = False

    @property
    def is_expert(self) -> bool:
        return self.expert_id is not None

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def _norm_bias(cfg: ModelConfig, key: str) -> List[dict]:
    """LayerNorm's bias next to a norm weight (TransformerEngine / Megatron names); none under RMSNorm."""
    if cfg.normalization != "LayerNorm":
        return []
    bkey = key[:-len("weight")] + "bias"
    return [dict(key=bkey, shape=(cfg.hidden_size,), sp_partial=True, weight_decay=False, init="zeros")]


def _layer_params(cfg: ModelConfig) -> List[dict]:
    h = cfg.hidden_size
    out = [
        dict(key="self_attention.linear_qkv.layer_norm_weight", shape=(h,), sp_partial=True, weight_decay=False,
             init="ones"),
        *_norm_bias(cfg, "self_attention.linear_qkv.layer_norm_weight"),
        dict(key="self_attention.linear_qkv.weight", shape=(cfg.qkv_rows, h), tp_dim=0),
        dict(key="self_attention.linear_proj.weight", shape=(h, cfg.num_attention_heads * cfg.head_dim), tp_dim=1),
    ]
    if cfg.is_moe:
        f = cfg.moe_ffn_hidden_size
        out.append(dict(key="pre_mlp_layernorm.weight", shape=(h,), sp_partial=True, weight_decay=False,
                        init="ones"))
        out += _norm_bias(cfg, "pre_mlp_layernorm.weight")
        out.append(dict(key="mlp.router.weight", shape=(cfg.num_experts, h), sp_partial=True))
        for e in range(cfg.num_experts):
            out.append(dict(key="mlp.experts.linear_fc1.weight", shape=(2 * f, h), tp_dim=0, tp_kind="swiglu",
                            expert_id=e, name=f"mlp.experts.local_experts.{e}.linear_fc1.weight"))
            out.append(dict(key="mlp.experts.linear_fc2.weight", shape=(h, f), tp_dim=1, expert_id=e,
                            name=f"mlp.experts.local_experts.{e}.linear_fc2.weight"))
    else:
        f = cfg.ffn_hidden_size
        out.append(dict(key="mlp.linear_fc1.layer_norm_weight", shape=(h,), sp_partial=True, weight_decay=False,
                        init="ones"))
        out += _norm_bias(cfg, "mlp.linear_fc1.layer_norm_weight")
        out.append(dict(key="mlp.linear_fc1.weight", shape=(2 * f, h), tp_dim=0, tp_kind="swiglu"))
        out.append(dict(key="mlp.linear_fc2.weight", shape=(h, f), tp_dim=1))
    return out


def build_virtual_params(cfg: ModelConfig) -> List[VParam]:
    """Global parameter list in canonical (forward / transfer) order."""
    h, v = cfg.hidden_size, cfg.padded_vocab_size
    vps: List[VParam] = []

    def add(**kw):
        vps.append(VParam(index=len(vps), **kw))

    add(name="embedding.word_embeddings.weight", shape=(v, h), tp_dim=0, stage_kind=PRE,
        local_key="embedding.word_embeddings.weight", tied_head=not cfg.untie_embeddings_and_output_weights)
    for layer in range(cfg.num_layers):
        for p in _layer_params(cfg):
            name = p.pop("name", p["key"])
            key = p.pop("key")
            add(name=f"decoder.layers.{layer}.{name}", layer_id=layer, stage_kind=LAYER, local_key=key, **p)
    add(name="decoder.final_layernorm.weight", shape=(h,), stage_kind=POST, sp_partial=True, weight_decay=False,
        init="ones", local_key="decoder.final_layernorm.weight")
    if cfg.normalization == "LayerNorm":
        add(name="decoder.final_layernorm.bias", shape=(h,), stage_kind=POST, sp_partial=True, weight_decay=False,
            init="zeros", local_key="decoder.final_layernorm.bias")
    if cfg.untie_embeddings_and_output_weights:
        add(name="output_layer.weight", shape=(v, h), tp_dim=0, stage_kind=POST, local_key="output_layer.weight")
    return vps


@dataclass
class LocalParam:
    """A model parameter as stored on one rank under one strategy."""

    name: str  # local name (local layer index), Megatron legacy-checkpoint style
    key: str  # layer-relative key (or global name for pre/post params)
    shape: Tuple[int, ...]
    is_expert: bool
    layer_local: Optional[int]
    weight_decay: bool
    sp_partial: bool
    # (virtual param, element offset of the virtual param's local shard inside this tensor)
    members: List[Tuple[VParam, int]] = field(default_factory=list)
    # tied word embedding: its gradient is summed over the embedding group (first and last pipeline stage)
    # before the DP reduction; ``replica`` marks the last stage's copy, which the gradient norm skips
    tied: bool = False
    replica: bool = False

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def stage_of(vp: VParam, cfg: ModelConfig, pp: int) -> int:
    if vp.stage_kind == PRE:
        return 0
    if vp.stage_kind == POST:
        return pp - 1
    return vp.layer_id // (cfg.num_layers // pp)


def stages_of(vp: VParam, cfg: ModelConfig, pp: int) -> Tuple[int, ...]:
    """Every pipeline stage that holds ``vp``: a tied word embedding is held by the first stage and, as the
    output layer, by the last (Megatron keeps the same pair of copies and sums their gradients)."""
    st = stage_of(vp, cfg, pp)
    if vp.tied_head and pp > 1:
        return (st, pp - 1)
    return (st,)


def tp_local_shape(vp: VParam, tp: int) -> Tuple[int, ...]:
    if vp.tp_dim is None or tp == 1:
        return vp.shape
    s = list(vp.shape)
    assert s[vp.tp_dim] % tp == 0, f"{vp.name}: dim {vp.tp_dim} of {vp.shape} not divisible by TP {tp}"
    s[vp.tp_dim] //= tp
    return tuple(s)


def local_params(cfg: ModelConfig, vps: List[VParam], strategy, rank: int) -> List[LocalParam]:
    """Model parameters of ``rank`` under ``strategy`` in forward order (pure function)."""
    c = strategy.coords(rank)
    pp = strategy.pipeline_model_parallel_size
    per_stage = cfg.num_layers // pp
    out: List[LocalParam] = []
    stacked: Dict[Tuple[int, str], LocalParam] = {}
    head_copy = None
    for vp in vps:
        if vp.tied_head and pp > 1 and c["pp"] == pp - 1:
            # the last stage's copy of the tied embedding, used as the output layer (after the final norm)
            head_copy = LocalParam(name="output_layer.weight", key="output_layer.weight",
                                   shape=tp_local_shape(vp, strategy.tensor_model_parallel_size), is_expert=False,
                                   layer_local=None, weight_decay=vp.weight_decay, sp_partial=False,
                                   members=[(vp, 0)], tied=True, replica=True)
            continue
        if stage_of(vp, cfg, pp) != c["pp"]:
            continue
        if vp.is_expert:
            e_loc_n = strategy.expert_num_per_ep_rank
            if vp.expert_id // e_loc_n != c["ep"]:
                continue
            e_loc = vp.expert_id % e_loc_n
            shp = tp_local_shape(vp, strategy.expert_tensor_parallel_size)
            key = (vp.layer_id, vp.local_key)
            lp = stacked.get(key)
            if lp is None:
                ll = vp.layer_id - c["pp"] * per_stage
                lp = LocalParam(name=f"decoder.layers.{ll}.{vp.local_key}", key=vp.local_key,
                                shape=(e_loc_n,) + shp, is_expert=True, layer_local=ll,
                                weight_decay=vp.weight_decay, sp_partial=False)
                stacked[key] = lp
                out.append(lp)
            n = 1
            for s in shp:
                n *= s
            lp.members.append((vp, e_loc * n))
            continue
        shp = tp_local_shape(vp, strategy.tensor_model_parallel_size)
        if vp.stage_kind == LAYER:
            ll = vp.layer_id - c["pp"] * per_stage
            name = f"decoder.layers.{ll}.{vp.local_key}"
        else:
            ll = None
            name = vp.name
        out.append(LocalParam(name=name, key=vp.local_key, shape=shp, is_expert=False, layer_local=ll,
                              weight_decay=vp.weight_decay, sp_partial=vp.sp_partial, members=[(vp, 0)],
                              tied=vp.tied_head))
    if head_copy is not None:
        out.append(head_copy)
    return out


# ---------------------------------------------------------------------------------------------------------
# TP index maps: which global rows / columns a TP rank holds.
def tp_row_blocks(vp: VParam, tp: int, tp_rank: int) -> List[Tuple[int, int, int]]:
    """For a dim-0 split: list of (global_row_start, local_row_start, n_rows) blocks held by ``tp_rank``."""
    rows = vp.shape[0]
    if vp.tp_dim != 0 or tp == 1:
        return [(0, 0, rows)]
    if vp.tp_kind == "swiglu":
        half = rows // 2
        n = half // tp
        return [(tp_rank * n, 0, n), (half + tp_rank * n, n, n)]
    n = rows // tp
    return [(tp_rank * n, 0, n)]


def tp_col_offset(vp: VParam, tp: int, tp_rank: int) -> int:
    if vp.tp_dim != 1 or tp == 1:
        return 0
    return tp_rank * (vp.shape[1] // tp)
