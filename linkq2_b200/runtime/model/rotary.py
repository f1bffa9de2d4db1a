"""Rotary position embedding, half-split ("neox") layout, fp32 rotation:
``qslab/runtime/model/rotary.py:12-16,83-111`` without the YaRN extension."""
from __future__ import annotations

import torch
from torch import nn


def apply_rotary_emb(x, cos, sin):
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_size: int, max_position: int, base: float, scaling: dict | None = None,
                 device=None):
        super().__init__()
        if scaling:
            raise NotImplementedError("rope scaling is outside the W4A16/KV4 hot path of this package")
        inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float, device="cpu") / head_size))
        freqs = torch.einsum("i,j -> ij", torch.arange(max_position, dtype=torch.float, device="cpu"), inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1).to(device or "cpu")
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def forward(self, positions, query, key):
        cos, sin = self.cos_sin_cache[positions].chunk(2, dim=-1)
        return apply_rotary_emb(query, cos, sin), apply_rotary_emb(key, cos, sin)
