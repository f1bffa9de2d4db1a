"""One attention layer's interface into the int4 paged KV pool.

Mirror of ``PagedAttention`` (``qslab/runtime/model/attention.py:21-144``) for
the KV4 cache: SmoothAttention scaling, store before attention, paged decode /
verify through the KV4 kernels, and prefill over the fp16 rows of the step plus
the pool-resident prefix.  The reference restores the prefix to fp16 and runs
both through the flash-attn wheel (``attention.py:38-56,121-131``); here the
prefix is read as int4 by the KV4 prefix kernel and merged with the attention
over the step's own rows.  ``num_heads`` / ``num_kv_heads`` are this rank's shard.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from linkq2_b200.kernels.kv4 import paged_attention_decode, store_kv_quant
from linkq2_b200.kernels.kv4.ops import chunk_attention, paged_attention_prefix
from linkq2_b200.runtime.model.context import get_context

LONG_PROMPT = 256     # rows of one sequence in one step beyond which torch's fused attention takes over


class PagedAttention(nn.Module):
    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int,
                 block_n: int = 128, v_group: int = 64):
        super().__init__()
        self.num_heads, self.head_dim, self.scale = num_heads, head_dim, scale
        self.num_kv_heads = num_kv_heads
        self.block_n, self.v_group = block_n, v_group
        self.k_cache = self.v_cache = None      # (packed, scales) tuples
        self.kv_cache_dtype = 'kv4'
        self.lam = None                         # [H_kv, D] SmoothAttention
        self.lam_q = None                       # [H_q, D] expanded over each GQA group

    def set_smooth_lambda(self, lam: torch.Tensor):
        """``lam [H_kv, D]`` from the calibration file, kept in fp16 (the dtype the
        reference multiplies in, attention.py:76-77)."""
        self.lam = lam.to(torch.float16).contiguous()
        rep = self.num_heads // self.num_kv_heads
        self.lam_q = self.lam.repeat_interleave(rep, dim=0).contiguous()

    def _prefill(self, ctx, q, k, v):
        """Attention of the step's new rows: over themselves in fp16 (``chunk_attention``) and,
        for sequences with rows already in the pool, over that prefix read as int4 by the KV4
        prefix kernel; the first kernel merges the two parts by their softmax weights.  Replaces
        materialize + cat + flash-attn (``qslab/runtime/model/attention.py:38-56,119-131``).
        Only a prompt of more than 256 rows without prefix still goes through torch's fused
        attention, which is what the reference uses there too."""
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        pre = pre_lse = None
        if ctx.prefix_rows is not None:
            pre, pre_lse = paged_attention_prefix(
                q.index_select(0, ctx.prefix_rows), self.k_cache, self.v_cache, ctx.prefix_tables, ctx.prefix_lens,
                block_n=self.block_n, num_kv_heads=self.num_kv_heads, v_group=self.v_group,
                rows=ctx.prefix_rows.numel() // ctx.prefix_lens.numel())
        chunk_attention(q, k, v, ctx.chunk_first, ctx.chunk_prefix, pre, pre_lse, out)
        for cached, q0, q1 in ctx.prefix_plan:
            if cached == 0 and q1 - q0 > LONG_PROMPT:
                o = F.scaled_dot_product_attention(
                    q[q0:q1].transpose(0, 1).unsqueeze(0), k[q0:q1].transpose(0, 1).unsqueeze(0),
                    v[q0:q1].transpose(0, 1).unsqueeze(0), is_causal=True, scale=self.scale, enable_gqa=True)
                out[q0:q1] = o.squeeze(0).transpose(0, 1)
        return out

    def attend(self, q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor):
        """Attention for inputs that the fused pre-attention kernel has already
        rotated, scaled and written to the pool: paged decode / verify, or
        prefill over the step's fp16 rows plus the restored prefix."""
        ctx = get_context()
        if ctx.is_prefill:
            return self._prefill(ctx, q.view(-1, self.num_heads, self.head_dim),
                                 k.view(-1, self.num_kv_heads, self.head_dim),
                                 v.view(-1, self.num_kv_heads, self.head_dim))
        return paged_attention_decode(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens,
                                      block_n=self.block_n, num_kv_heads=self.num_kv_heads,
                                      k_scale=self.k_cache[1], v_group=self.v_group, verify_m=ctx.verify_m)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        ctx = get_context()
        if self.kv_cache_dtype != 'kv4':
            raise NotImplementedError("this package implements the KV4 cache path only")
        if self.lam is not None:
            q = q * self.lam_q.to(q.dtype)
            k = k / self.lam.to(k.dtype)
        k_cache, v_cache = self.k_cache, self.v_cache
        # store first: decode's context_lens includes the token being processed
        if k_cache is not None and v_cache is not None and k.shape[0] > 0:
            store_kv_quant(k.view(-1, self.num_kv_heads, self.head_dim),
                           v.view(-1, self.num_kv_heads, self.head_dim),
                           k_cache, v_cache, ctx.slot_mapping.view(-1), v_group=self.v_group)
        if ctx.is_prefill:
            return self._prefill(ctx, q.view(-1, self.num_heads, self.head_dim),
                                 k.view(-1, self.num_kv_heads, self.head_dim),
                                 v.view(-1, self.num_kv_heads, self.head_dim))
        assert k_cache is not None and v_cache is not None
        return paged_attention_decode(q, k_cache, v_cache, ctx.block_tables, ctx.context_lens,
                                      block_n=self.block_n, num_kv_heads=self.num_kv_heads,
                                      k_scale=k_cache[1], v_group=self.v_group, verify_m=ctx.verify_m)
