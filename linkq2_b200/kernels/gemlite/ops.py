"""``linear(x, packed, scales, zeros, meta)`` — the launch interface of the
reference's W4A16 kernels (``qslab/kernels/gemlite/ops.py:10-15``) backed by the
sm_100a kernels of this package."""
from __future__ import annotations

import torch

from linkq2_b200 import _lib, _workspace


def set_constant_weights(enabled: bool) -> bool:
    """Declare the quantized weights constant (``lq2_w4a16_set_constant_weights``): ``linear``
    may then start fetching ``packed``/``scales``/``zeros`` before the previous kernel of the
    stream has finished.  Returns the previous setting.  Launches recorded into a CUDA graph
    keep the setting they were captured with."""
    return bool(_lib.lib.lq2_w4a16_set_constant_weights(1 if enabled else 0))


def can_push(rows: int, n: int, exchange) -> bool:
    """Shapes for which ``linear(..., push_to=exchange)`` exists: the tcgen05 kernel's pushed
    reduction (8 < rows <= 64) and a message that fits the exchange buffer."""
    return exchange is not None and 8 < rows <= 64 and rows * n * 2 <= exchange.max_bytes


def linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
           meta, *, gate_up_silu: bool = False, push_to=None) -> torch.Tensor:
    """``x [..., K] fp16`` times the dequantised ``[K, N]`` weight -> ``[..., N] fp16``.

    ``packed [K/8, N] int32``, ``scales [K/G, N] fp16``; ``zeros`` is either the
    ``[K/G, N] fp16`` zero-point table or a one-element tensor, which selects
    the symmetric scalar zero 8 exactly as ``zeros.numel() == 1`` does in the
    reference (``triton_kernels/gemv_revsplitK_A16fWnO16f_int32packing.py:376``).
    ``meta`` is the 12-tuple built by ``from_quantized``; only its bit width,
    group size and group mode are read.

    ``gate_up_silu`` (no counterpart in the reference's signature): the buffers hold a
    gate and an up projection with their columns interleaved in blocks of four
    (``B200Linear.fuse_gate_up``); the result is ``silu(gate(x)) * up(x)``, ``N / 2`` wide
    (``lq2_w4a16_gate_up_silu``).

    ``push_to`` (a ``PeerExchange``): the projection is row-split under tensor parallelism;
    besides returning this rank's partial sum the kernel sends it to the peers' exchange
    buffers (``lq2_w4a16_linear_push``).  Only for ``can_push(rows, n, exchange)`` shapes;
    the next exchange call must be ``rmsnorm_allreduce(..., pushed=True)`` on the result.
    """
    if meta[0] != 4 or meta[9] != 3:
        raise ValueError("only 4-bit weights with (u - zero) * scale dequantisation are supported")
    group = int(meta[1])
    if x.dtype != torch.float16:
        raise TypeError(f"the B200 W4A16 kernels compute in fp16, got {x.dtype}")
    if not x.is_cuda:
        raise RuntimeError("linkq2_b200 operators run on CUDA tensors only")
    k8, n = packed.shape
    k = k8 * 8
    if x.shape[-1] != k:
        raise ValueError(f"expected input width {k}, got {x.shape[-1]}")
    if gate_up_silu and n % 64:
        raise ValueError("gate_up_silu needs a multiple of 64 fused columns")
    n_out = n // 2 if gate_up_silu else n
    shape = x.shape[:-1] + (n_out,)
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    m = x2.shape[0]
    y = torch.empty((m, n_out), dtype=torch.float16, device=x.device)
    if m == 0:
        return y.view(shape)
    zero_ptr = None if zeros.numel() == 1 else zeros.data_ptr()
    with torch.cuda.device(x.device):
        need = _lib.lib.lq2_w4a16_workspace_bytes(m, n, k)
        ws = _workspace.get("w4a16", need, x.device) if need else None
        stream = torch.cuda.current_stream().cuda_stream
        if push_to is not None:
            status = _lib.lib.lq2_w4a16_linear_push(
                x2.data_ptr(), x2.stride(0), packed.data_ptr(), scales.data_ptr(), zero_ptr, y.data_ptr(),
                m, n, k, group, push_to.table, push_to.rank, push_to.world, push_to.max_bytes, stream)
            _lib.check(status, "lq2_w4a16_linear_push")
            _lib.count()
            return y.view(shape)
        entry = _lib.lib.lq2_w4a16_gate_up_silu if gate_up_silu else _lib.lib.lq2_w4a16_linear
        status = entry(
            x2.data_ptr(), x2.stride(0), packed.data_ptr(), scales.data_ptr(), zero_ptr, y.data_ptr(),
            m, n, k, group, ws.data_ptr() if need else None, ws.numel() if need else 0, stream)
    _lib.check(status, "lq2_w4a16_gate_up_silu" if gate_up_silu else "lq2_w4a16_linear")
    _lib.count()
    return y.view(shape)
