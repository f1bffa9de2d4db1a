"""int4 weight packing on the GPU (``qslab/kernels/gemlite/bitpack.py:96-125``)."""
from __future__ import annotations

import torch

from linkq2_b200 import _lib


def pack_w4(values: torch.Tensor, symmetric: bool) -> torch.Tensor:
    """``values [N, K]`` int8/uint8 checkpoint integers on a CUDA device ->
    ``packed [K/8, N] int32`` contiguous; symmetric checkpoints (-8..7) are
    offset by +8 first (``qslab/runtime/backends/gemlite.py:22-25``)."""
    if values.dim() != 2 or values.dtype not in (torch.int8, torch.uint8):
        raise TypeError("values must be a 2-D int8/uint8 tensor")
    if not values.is_cuda:
        raise RuntimeError("pack_w4 runs on the GPU; move values to a CUDA device")
    n, k = values.shape
    if k % 8:
        raise ValueError(f"unsupported W4A16 shape: K={k} is not a multiple of 8")
    values = values.contiguous()
    packed = torch.empty((k // 8, n), dtype=torch.int32, device=values.device)
    with torch.cuda.device(values.device):
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib.lq2_w4_pack(values.data_ptr(), 8 if symmetric else 0, packed.data_ptr(),
                                        n, k, stream), "lq2_w4_pack")
    _lib.count()
    return packed


def pack_weights_over_cols(codes: torch.Tensor, W_nbits: int = 4, packing_bitwidth: int = 32,
                           transpose: bool = True):
    """Call-compatible stand-in for ``pack_weights_over_cols_triton`` for the one
    configuration the runtime uses (4-bit codes, 32-bit words, transposed):
    ``codes [N, K] uint8`` in 0..15 -> ``([K/8, N] int32, 8)``."""
    if (W_nbits, packing_bitwidth, transpose) != (4, 32, True):
        raise ValueError("only 4-bit codes in transposed 32-bit words are supported")
    return pack_w4(codes.to(torch.uint8), symmetric=False), 8
