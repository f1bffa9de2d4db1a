"""Scratch buffers for the split-K / split-KV kernels.

The kernels need a zero-initialised scratch buffer that they leave zeroed
again; one buffer per (device, stream, kind) is kept and grown on demand.  A
buffer that has been handed out is never freed: a captured CUDA graph may hold
its address.  Inside stream capture a missing or too-small buffer is allocated
from the capturing pool and not cached (the zero fill becomes a graph node), the
same way the reference allocates its split partials inside capture
(``qslab/kernels/kv4/paged_attention.py:132``).
"""
from __future__ import annotations

import torch

_cache: dict[tuple, torch.Tensor] = {}
_retired: list[torch.Tensor] = []


def get(kind: str, nbytes: int, device: torch.device) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = (kind, device.index, stream.cuda_stream)
    buf = _cache.get(key)
    if buf is not None and buf.numel() >= nbytes:
        return buf
    if torch.cuda.is_current_stream_capturing():
        return torch.zeros(nbytes, dtype=torch.uint8, device=device)
    if buf is not None:
        _retired.append(buf)
    buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
    _cache[key] = buf
    return buf
