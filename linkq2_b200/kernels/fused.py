"""Fused elementwise steps of a decoder layer (RMSNorm with residual, SiLU * up,
and q/k-norm + RoPE + SmoothAttention scaling + KV4 store).  The reference runs
these as eager torch ops (``qslab/runtime/model/primitives.py:15-36``,
``qwen3.py:49-51,64``, ``rotary.py:12-16``, ``attention.py:72-77,102-110``)."""
from __future__ import annotations

import torch

from linkq2_b200 import _lib


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """``x [..., hidden] fp16``.  Without ``residual`` returns the normalised
    tensor; with it returns ``(normalised, x + residual)``."""
    if x.dtype != torch.float16 or not x.is_cuda:
        raise TypeError("rmsnorm runs on CUDA fp16 tensors")
    hidden = x.shape[-1]
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    out = torch.empty((rows, hidden), dtype=torch.float16, device=x.device)
    res_in = res_out = None
    if residual is not None:
        res_in = residual.reshape(-1, hidden)
        res_in = res_in if res_in.is_contiguous() else res_in.contiguous()
        res_out = torch.empty_like(out)
    with torch.cuda.device(x.device):
        status = _lib.lib.lq2_rmsnorm(x2.data_ptr(), x2.stride(0), None if res_in is None else res_in.data_ptr(),
                                      weight.data_ptr(), out.data_ptr(),
                                      None if res_out is None else res_out.data_ptr(), rows, hidden, eps, _stream(x))
    _lib.check(status, "lq2_rmsnorm")
    _lib.count()
    out = out.view(x.shape)
    return out if residual is None else (out, res_out.view(x.shape))


def rmsnorm_allreduce(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor, exchange,
                      pushed: bool = False):
    """``rmsnorm(all_reduce(x), weight, eps, residual)`` in one launch: ``x`` is this
    rank's partial sum; the exchange runs over peer memory inside the norm kernel
    (``exchange``: the ``PeerExchange`` of the tensor-parallel group).  Returns
    ``(normalised, all_reduce(x) + residual)``.  ``pushed``: the projection that produced
    ``x`` has already sent it to the peers (``linear(..., push_to=exchange)``); only gather."""
    if x.dtype != torch.float16 or not x.is_cuda:
        raise TypeError("rmsnorm_allreduce runs on CUDA fp16 tensors")
    hidden = x.shape[-1]
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    res_in = residual.reshape(-1, hidden)
    res_in = res_in if res_in.is_contiguous() else res_in.contiguous()
    out = torch.empty((rows, hidden), dtype=torch.float16, device=x.device)
    res_out = torch.empty_like(out)
    with torch.cuda.device(x.device):
        entry = _lib.lib.lq2_rmsnorm_allreduce_pushed if pushed else _lib.lib.lq2_rmsnorm_allreduce
        status = entry(
            x2.data_ptr(), x2.stride(0), res_in.data_ptr(), weight.data_ptr(), out.data_ptr(), res_out.data_ptr(),
            rows, hidden, eps, exchange.table, exchange.rank, exchange.world, exchange.max_bytes, _stream(x))
    _lib.check(status, "lq2_rmsnorm_allreduce")
    _lib.count()
    return out.view(x.shape), res_out.view(x.shape)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``[rows, width] fp16`` tensors (row strides allowed)."""
    if gate.dtype != torch.float16 or not gate.is_cuda:
        raise TypeError("silu_mul runs on CUDA fp16 tensors")
    width = gate.shape[-1]
    g2, u2 = gate.reshape(-1, width), up.reshape(-1, width)
    if g2.stride(-1) != 1 or g2.stride(0) % 8 or g2.data_ptr() % 16:
        g2 = g2.contiguous()
    if u2.stride(-1) != 1 or u2.stride(0) % 8 or u2.data_ptr() % 16:
        u2 = u2.contiguous()
    out = torch.empty((g2.shape[0], width), dtype=torch.float16, device=gate.device)
    with torch.cuda.device(gate.device):
        status = _lib.lib.lq2_silu_mul(g2.data_ptr(), g2.stride(0), u2.data_ptr(), u2.stride(0), out.data_ptr(),
                                       g2.shape[0], width, _stream(gate))
    _lib.check(status, "lq2_silu_mul")
    _lib.count()
    return out.view(gate.shape)


def pre_attention(q, k, v, q_weight, k_weight, cos_sin, positions, eps, *, lam_q=None, lam_k=None,
                  k_cache=None, v_cache=None, slot_mapping=None, v_group=64, want_k=False):
    """``q [T, HQ, D]``, ``k, v [T, HKV, D]`` fp16 (token-strided views allowed) ->
    ``(q_out, k_out | None)``; when the caches and ``slot_mapping`` are given the
    rotated keys and the values are quantized into the pool in the same launch."""
    t, hq, d = q.shape
    hkv = k.shape[1]
    for name, x in (("q", q), ("k", k), ("v", v)):
        if x.dtype != torch.float16 or not x.is_cuda:
            raise TypeError("pre_attention runs on CUDA fp16 tensors")
        if x.stride(2) != 1 or x.stride(1) != d:
            raise ValueError(f"{name} must have unit channel stride and head stride D")
    q_out = torch.empty((t, hq, d), dtype=torch.float16, device=q.device)
    k_out = torch.empty((t, hkv, d), dtype=torch.float16, device=q.device) if want_k else None
    store = k_cache is not None and slot_mapping is not None
    kq = ks = vq = vs = slots = None
    num_slots = 0
    if store:
        (kq, ks), (vq, vs) = k_cache, v_cache
        if ks.dim() != 2 or tuple(ks.shape) != (hkv, d):
            raise ValueError(f"K scale must be the static [{hkv}, {d}] fp16 table, got {tuple(ks.shape)}")
        slots = slot_mapping.to(torch.int32).contiguous()
        num_slots = kq.shape[0]
    cs = cos_sin.reshape(-1, d)
    pos = positions.to(torch.int64).contiguous()
    ptr = lambda x: None if x is None else x.data_ptr()
    with torch.cuda.device(q.device):
        status = _lib.lib.lq2_pre_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0),
            q_weight.data_ptr(), k_weight.data_ptr(), cs.data_ptr(), pos.data_ptr(), ptr(lam_q), ptr(lam_k),
            q_out.data_ptr(), ptr(k_out), ptr(kq), ptr(ks), ptr(vq), ptr(vs), ptr(slots),
            t, hq, hkv, d, v_group, num_slots, eps, _stream(q))
    _lib.check(status, "lq2_pre_attention")
    _lib.count()
    return q_out, k_out
