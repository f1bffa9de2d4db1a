"""Qwen3 decoder with W4-swappable projections, int4 paged attention and a
tensor-parallel split.

Layer graph and module names follow ``qslab/runtime/model/qwen3.py:18-137`` (and
the HF checkpoint): separate q/k/v/gate/up projections, q/k RMSNorm, RoPE,
residual-fused RMSNorm.  Under tensor parallelism every rank holds
``heads / t`` query heads, ``kv_heads / t`` KV heads and ``intermediate / t``
MLP channels; ``o_proj`` and ``down_proj`` produce partial sums that are
all-reduced.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from linkq2_b200.kernels.fused import pre_attention, silu_mul
from linkq2_b200.runtime.model.attention import PagedAttention
from linkq2_b200.runtime.model.context import get_context
from linkq2_b200.runtime.model.primitives import Linear, LMHead, RMSNorm, VocabEmbedding
from linkq2_b200.runtime.model.rotary import RotaryEmbedding
from linkq2_b200.runtime.parallel import get_tp


@dataclass
class ModelConfig:
    """The fields of a HF ``Qwen3Config`` this runtime reads."""
    vocab_size: int = 151936
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False

    @classmethod
    def from_dict(cls, cfg: dict) -> "ModelConfig":
        fields = {f: cfg[f] for f in cls.__dataclass_fields__ if f in cfg}
        if "head_dim" not in fields:
            fields["head_dim"] = cfg["hidden_size"] // cfg["num_attention_heads"]
        if "rope_theta" not in fields and isinstance(cfg.get("rope_parameters"), dict):
            fields["rope_theta"] = cfg["rope_parameters"].get("rope_theta", 1e6)
        return cls(**fields)

    @classmethod
    def qwen3_8b(cls):
        return cls()

    @classmethod
    def qwen3_1p7b(cls):
        return cls(hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                   num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                   tie_word_embeddings=True)


def _fuse(layers, gate_up=False):
    """Fused W4 projection for layers sharing their input, or None when they are
    not packed W4 layers or carry AWQ input scales (the reason the reference keeps
    them apart, ``qslab/runtime/model/qwen3.py:3-5``).  ``gate_up``: the pair is fused
    together with the SiLU * up that follows it."""
    from linkq2_b200.runtime.backends.b200 import B200Linear
    if not all(isinstance(l, B200Linear) and l.input_scale is None for l in layers):
        return None
    if gate_up and layers[0].out_features % 32 == 0 and os.environ.get("LQ2_FUSE_SILU", "1") != "0":
        return B200Linear.fuse_gate_up(*layers)
    return B200Linear.fuse_columns(layers)


class Qwen3Attention(nn.Module):
    def __init__(self, config: ModelConfig, rope: RotaryEmbedding):
        super().__init__()
        tp = get_tp()
        self.tp = tp
        self.num_heads = config.num_attention_heads // tp.size
        self.num_kv_heads = config.num_key_value_heads // tp.size
        self.head_dim = config.head_dim
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.q_proj = Linear(config.hidden_size, self.q_size)
        self.k_proj = Linear(config.hidden_size, self.kv_size)
        self.v_proj = Linear(config.hidden_size, self.kv_size)
        self.o_proj = Linear(self.q_size, config.hidden_size)
        self.qkv_proj = None
        self.rotary_emb = rope
        self.attn = PagedAttention(self.num_heads, self.head_dim, self.head_dim ** -0.5, self.num_kv_heads)
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)

    def fuse(self):
        """Replace q/k/v by one projection when the checkpoint allows it."""
        self.qkv_proj = _fuse([self.q_proj, self.k_proj, self.v_proj])
        if self.qkv_proj is not None:
            self.q_proj = self.k_proj = self.v_proj = None

    def forward(self, positions, hidden_states):
        if self.qkv_proj is not None:
            q, k, v = self.qkv_proj(hidden_states).split([self.q_size, self.kv_size, self.kv_size], dim=-1)
            q = q.unflatten(-1, (self.num_heads, self.head_dim))
            k = k.unflatten(-1, (self.num_kv_heads, self.head_dim))
            v = v.unflatten(-1, (self.num_kv_heads, self.head_dim))
        else:
            q = self.q_proj(hidden_states).view(-1, self.num_heads, self.head_dim)
            k = self.k_proj(hidden_states).view(-1, self.num_kv_heads, self.head_dim)
            v = self.v_proj(hidden_states).view(-1, self.num_kv_heads, self.head_dim)
        # q/k norm, RoPE, SmoothAttention scaling and the KV4 store in one launch
        ctx = get_context()
        attn = self.attn
        store = attn.k_cache is not None and ctx.slot_mapping is not None
        q, k = pre_attention(q, k, v, self.q_norm.weight, self.k_norm.weight, self.rotary_emb.cos_sin_cache,
                             positions, self.q_norm.eps, lam_q=attn.lam_q, lam_k=attn.lam,
                             k_cache=attn.k_cache if store else None, v_cache=attn.v_cache if store else None,
                             slot_mapping=ctx.slot_mapping if store else None, v_group=attn.v_group,
                             want_k=ctx.is_prefill)
        o = attn.attend(q, k, v)
        return self.tp.project_reduce_or_defer(self.o_proj, o.flatten(1, -1))


class Qwen3MLP(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        tp = get_tp()
        self.tp = tp
        inter = config.intermediate_size // tp.size
        self.gate_proj = Linear(config.hidden_size, inter)
        self.up_proj = Linear(config.hidden_size, inter)
        self.down_proj = Linear(inter, config.hidden_size)
        self.gate_up_proj = None

    def fuse(self):
        """Replace gate/up by one projection with the activation in its epilogue when the
        checkpoint allows it."""
        self.gate_up_proj = _fuse([self.gate_proj, self.up_proj], gate_up=True)
        if self.gate_up_proj is not None:
            self.gate_proj = self.up_proj = None

    def forward(self, x):
        if self.gate_up_proj is not None and getattr(self.gate_up_proj, "gate_up_silu", False):
            hidden = self.gate_up_proj(x)                   # silu(gate(x)) * up(x)
        elif self.gate_up_proj is not None:
            hidden = silu_mul(*self.gate_up_proj(x).chunk(2, dim=-1))
        else:
            hidden = silu_mul(self.gate_proj(x), self.up_proj(x))
        return self.tp.project_reduce_or_defer(self.down_proj, hidden)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, config: ModelConfig, rope: RotaryEmbedding):
        super().__init__()
        self.self_attn = Qwen3Attention(config, rope)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, positions, hidden_states, residual, deferred=False):
        """``deferred``: ``hidden_states`` is the previous layer's MLP output before its
        tensor-parallel all-reduce, which the norm below then performs itself.  Returns
        ``(mlp_out, residual, deferred)`` in the same convention."""
        if residual is None:
            hidden_states, residual = self.input_layernorm(hidden_states), hidden_states
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual, deferred=deferred)
        hidden_states, deferred = self.self_attn(positions, hidden_states)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual, deferred=deferred)
        hidden_states, deferred = self.mlp(hidden_states)
        return hidden_states, residual, deferred


class Qwen3Model(nn.Module):
    def __init__(self, config: ModelConfig, max_position: int | None = None, device=None):
        super().__init__()
        rope = RotaryEmbedding(config.head_dim, max_position or config.max_position_embeddings,
                               config.rope_theta, device=device)
        self.embed_tokens = VocabEmbedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config, rope) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, input_ids, positions):
        hidden_states, residual, deferred = self.embed_tokens(input_ids), None, False
        for layer in self.layers:
            hidden_states, residual, deferred = layer(positions, hidden_states, residual, deferred)
        hidden_states, _ = self.norm(hidden_states, residual, deferred=deferred)
        return hidden_states


class Qwen3ForCausalLM(nn.Module):
    # module-name suffix -> how its weight is split across tensor-parallel ranks
    TP_SPLIT = {"q_proj": "column", "k_proj": "column", "v_proj": "column", "gate_proj": "column",
                "up_proj": "column", "o_proj": "row", "down_proj": "row"}

    def __init__(self, config: ModelConfig, max_position: int | None = None, device=None):
        super().__init__()
        self.config = config
        self.model = Qwen3Model(config, max_position, device)
        self.lm_head = LMHead(config.vocab_size, config.hidden_size)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.head_rows = None            # (first row, rows, vocabulary) once shard_head() has cut the head

    def fuse_projections(self):
        """Fuse q/k/v and gate/up of every layer into single W4 launches (a
        load-time layout step: buffers are concatenated along N, nothing is
        repacked).  Layers of AWQ checkpoints are left as they are."""
        for layer in self.model.layers:
            layer.self_attn.fuse()
            layer.mlp.fuse()
        return self

    def forward(self, input_ids, positions):
        return self.model(input_ids, positions)

    def shard_head(self):
        """Under tensor parallelism keep only this rank's slice of the vocabulary rows of an
        untied LM head (1.2 GB of fp16 at Qwen3-8B size, replicated otherwise).  A head tied to
        the embedding stays whole, because the embedding lookup needs every row, and is
        sliced as a view at use.  Replaces the replicated head of
        ``qslab/runtime/execute/model_runner.py:398``."""
        tp = get_tp()
        vocab = self.lm_head.weight.shape[0]
        if tp.size == 1 or vocab % tp.size or self.config.tie_word_embeddings or self.head_rows is not None:
            return self
        share = vocab // tp.size
        local = self.lm_head.weight.data[tp.rank * share:(tp.rank + 1) * share].clone()
        self.lm_head.weight = nn.Parameter(local, requires_grad=False)
        self.head_rows = (tp.rank * share, share, vocab)
        return self

    def _local_logits(self, hidden_states):
        """``(logits of this rank's vocabulary slice, first row of the slice, vocabulary size)``;
        the whole vocabulary when the head cannot be split evenly or there is one rank."""
        tp = get_tp()
        weight = self.lm_head.weight
        if self.head_rows is not None:
            first, _, vocab = self.head_rows
            return F.linear(hidden_states, weight), first, vocab
        vocab = weight.shape[0]
        if tp.size == 1 or vocab % tp.size or not dist.is_initialized():
            return self.lm_head(hidden_states), 0, vocab
        share = vocab // tp.size
        return F.linear(hidden_states, weight[tp.rank * share:(tp.rank + 1) * share]), tp.rank * share, vocab

    def compute_logits(self, hidden_states):
        """Logits over the whole vocabulary.  Under tensor parallelism each rank multiplies
        by its slice of the head only and the slices are gathered (``greedy_tokens`` avoids the
        gather when only the arg-max is wanted)."""
        tp = get_tp()
        local, _, vocab = self._local_logits(hidden_states)
        if local.shape[-1] == vocab:
            return local
        parts = torch.empty((tp.size,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(parts, local.contiguous(), group=tp.group)
        return parts.movedim(0, -2).reshape(*local.shape[:-1], vocab)

    def greedy_tokens(self, hidden_states):
        """Arg-max token per row, equal to ``compute_logits(h).argmax(-1)`` (ties go to the lowest
        index).  Under tensor parallelism the ranks exchange one (value, index) pair per row
        instead of their logits: 8 bytes per row and rank against 2 * vocab / t."""
        tp = get_tp()
        local, first, vocab = self._local_logits(hidden_states)
        if local.shape[-1] == vocab:
            return local.argmax(dim=-1)
        value, index = local.max(dim=-1)                      # index of the first maximum
        pair = torch.stack([value.float(), (index + first).float()], dim=-1).contiguous()   # ids < 2**24: exact
        pairs = torch.empty((tp.size,) + tuple(pair.shape), dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(pairs, pair, group=tp.group)
        best = pairs[..., 0].argmax(dim=0, keepdim=True)      # first maximum: the lowest rank, so the lowest index
        return pairs[..., 1].gather(0, best).squeeze(0).long()
