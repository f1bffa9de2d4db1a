"""RMSNorm, dense Linear, embedding and LM head with the arithmetic of
``qslab/runtime/model/primitives.py:9-78`` (fp32 statistics, fp16 storage).
RMSNorm runs as one fused kernel; ``reference_forward`` is the reference's eager
expression, kept for the numerics tests."""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size), requires_grad=False)

    def forward(self, x, residual=None, deferred=False):
        """``deferred``: ``x`` is this rank's partial sum of a row-split projection;
        the tensor-parallel all-reduce is done inside the norm kernel."""
        from linkq2_b200.kernels.fused import rmsnorm, rmsnorm_allreduce
        if deferred:
            from linkq2_b200.runtime.parallel import get_tp
            return rmsnorm_allreduce(x, self.weight, self.eps, residual, get_tp().exchange, pushed=deferred == 2)
        return rmsnorm(x, self.weight, self.eps, residual)

    def reference_forward(self, x, residual=None):
        orig = x.dtype
        if residual is None:
            x = x.float()
            var = x.pow(2).mean(dim=-1, keepdim=True)
            return (x * torch.rsqrt(var + self.eps)).to(orig) * self.weight
        x = x.float() + residual.float()
        residual = x.to(orig)
        var = x.pow(2).mean(dim=-1, keepdim=True)
        return (x * torch.rsqrt(var + self.eps)).to(orig) * self.weight, residual


class Linear(nn.Module):
    def __init__(self, input_size: int, output_size: int):
        super().__init__()
        self.input_size, self.output_size = input_size, output_size
        self.weight = nn.Parameter(torch.empty(output_size, input_size), requires_grad=False)

    def forward(self, x):
        return F.linear(x, self.weight)


class VocabEmbedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim), requires_grad=False)

    def forward(self, x):
        return F.embedding(x, self.weight)


class LMHead(VocabEmbedding):
    def forward(self, x):
        return F.linear(x, self.weight)
