"""Per-step attention metadata shared by all layers; same fields and accessors
as ``qslab/runtime/model/context.py:5-36``."""
from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    # >1 marks a verify forward: M rows per sequence, row = seq*M + m
    verify_m: int = 1
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    # prefill: per sequence (cached rows, q_start, q_end); per query row the first row of its
    # sequence in this step (chunk_first) and where its prefix part will be found (chunk_prefix:
    # a row of the prefix kernel's output, -1 without prefix, -2 for rows of long prompts that go
    # through torch's fused attention instead).  For the sequences that have a prefix, the blocks
    # of query rows the KV4 prefix kernel works on: prefix_rows [blocks*r] (query row of every
    # block row, padded by repeating a row of the sequence), prefix_tables [blocks, width],
    # prefix_lens [blocks].
    prefix_plan: list | None = None
    chunk_first: torch.Tensor | None = None
    chunk_prefix: torch.Tensor | None = None
    prefix_rows: torch.Tensor | None = None
    prefix_tables: torch.Tensor | None = None
    prefix_lens: torch.Tensor | None = None


_CONTEXT = Context()


def get_context():
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None, verify_m=1,
                prefix_plan=None, chunk_first=None, chunk_prefix=None, prefix_rows=None, prefix_tables=None,
                prefix_lens=None):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, verify_m, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                       slot_mapping, context_lens, block_tables, prefix_plan, chunk_first, chunk_prefix,
                       prefix_rows, prefix_tables, prefix_lens)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
