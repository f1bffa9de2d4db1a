"""Python launchers of the KV4 kernels.  Caches are the reference's tuples:
``k_cache = (kq [S,HKV,D/8] uint32|int32, ks [HKV,D] fp16)``,
``v_cache = (vq [S,HKV,D/8], vs [S,HKV,D/v_group] fp16)``."""
from __future__ import annotations

import torch

from linkq2_b200 import _lib, _workspace


def _static_scale(ks: torch.Tensor, hkv: int, d: int) -> None:
    # The reference selects its static-table branch with ks.dim() == 2
    # (qslab/kernels/kv4/store.py:67); its other branch cannot be reached.
    if ks.dim() != 2 or tuple(ks.shape) != (hkv, d):
        raise ValueError(f"K scale must be the static [{hkv}, {d}] fp16 table, got {tuple(ks.shape)}")
    if ks.dtype != torch.float16:
        raise TypeError("K scale table must be fp16")


def store_kv_quant(k: torch.Tensor, v: torch.Tensor, k_cache, v_cache,
                   slot_mapping: torch.Tensor, v_group: int = 64) -> None:
    """Quantize ``k, v [T, HKV, D]`` into the pool at ``slot_mapping [T]``
    (``-1`` skips).  Same contract as ``qslab/kernels/kv4/store.py:58-68``; token
    strides are free (slices of a fused QKV buffer), head stride must be ``D``.
    fp16 is the runtime's type; like the reference's kernel, which converts what it
    loads to fp32 (``store.py:31,45``), fp32 tensors are quantized from their full
    precision and bf16 ones are widened to fp32 first."""
    t, h, d = k.shape
    kq, ks = k_cache
    vq, vs = v_cache
    floats = (torch.float16, torch.float32, torch.bfloat16)
    if k.dtype not in floats or v.dtype not in floats:
        raise TypeError("KV4 store takes floating-point keys and values")
    if not k.is_cuda:
        raise RuntimeError("linkq2_b200 operators run on CUDA tensors only")
    wide = k.dtype != torch.float16 or v.dtype != torch.float16
    if wide:
        k, v = k.float(), v.float()
    _static_scale(ks, h, d)
    if t == 0:
        return
    if k.stride(2) != 1 or k.stride(1) != d:
        k = k.contiguous()
    if v.stride(2) != 1 or v.stride(1) != d:
        v = v.contiguous()
    slots = slot_mapping.to(torch.int32)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    with torch.cuda.device(k.device):
        stream = torch.cuda.current_stream().cuda_stream
        entry = _lib.lib.lq2_kv4_store_f32 if wide else _lib.lib.lq2_kv4_store
        status = entry(
            k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), kq.data_ptr(), ks.data_ptr(),
            vq.data_ptr(), vs.data_ptr(), slots.data_ptr(), t, h, d, v_group, kq.shape[0], stream)
    _lib.check(status, "lq2_kv4_store")
    _lib.count()


def paged_attention_decode(q: torch.Tensor, k_cache, v_cache, block_tables: torch.Tensor,
                           context_lens: torch.Tensor, block_n: int = 128,
                           num_kv_heads: int | None = None, k_scale=None, v_group: int = 64,
                           verify_m: int = 1) -> torch.Tensor:
    """``q [rows, HQ, D] fp16 -> out [rows, HQ, D] fp16`` with ``rows = batch * verify_m``
    (``qslab/kernels/kv4/paged_attention.py:110-150``).  Row ``seq*verify_m + m``
    attends to positions ``[0, context_lens[seq] + m)``."""
    rows, hq, d = q.shape
    hkv = num_kv_heads if num_kv_heads is not None else hq
    kq, ks = k_cache
    vq, vs = v_cache
    if q.dtype != torch.float16:
        raise TypeError("KV4 attention takes fp16 queries")
    _static_scale(ks, hkv, d)
    out = torch.empty((rows, hq, d), dtype=torch.float16, device=q.device)
    if rows == 0:
        return out
    if rows % verify_m:
        raise ValueError("rows must be a multiple of verify_m")
    batch = rows // verify_m
    if q.stride(2) != 1 or q.stride(1) != d:
        q = q.contiguous()
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    bt = bt if bt.is_contiguous() else bt.contiguous()
    lens = context_lens if context_lens.dtype == torch.int32 else context_lens.to(torch.int32)
    max_blocks = bt.shape[1]
    args = (batch, verify_m, hq, hkv, d, block_n, max_blocks)
    with torch.cuda.device(q.device):
        need = _lib.lib.lq2_kv4_attention_workspace_bytes(*args)
        if need == 0:
            raise ValueError(f"unsupported KV4 attention shape: batch={batch} M={verify_m} HQ={hq} "
                             f"HKV={hkv} D={d} page={block_n} blocks={max_blocks}")
        ws = _workspace.get("kv4", need, q.device)
        stream = torch.cuda.current_stream().cuda_stream
        status = _lib.lib.lq2_kv4_attention(
            q.data_ptr(), q.stride(0), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
            bt.data_ptr(), lens.data_ptr(), out.data_ptr(), batch, verify_m, hq, hkv, d, block_n,
            max_blocks, v_group, kq.shape[0], ws.data_ptr(), ws.numel(), stream)
    _lib.check(status, "lq2_kv4_attention")
    _lib.count()
    return out


def paged_attention_prefix(q: torch.Tensor, k_cache, v_cache, block_tables: torch.Tensor,
                           prefix_lens: torch.Tensor, block_n: int = 128, num_kv_heads: int | None = None,
                           v_group: int = 64, rows: int = 16):
    """Attention of blocks of ``rows`` new query rows over the pool-resident prefix only:
    ``q [blocks*rows, HQ, D] fp16 -> (out [blocks*rows, HQ, D] fp16, lse [blocks*rows, HQ] fp32)``.
    Every row of block ``b`` attends to positions ``[0, prefix_lens[b])`` of ``block_tables[b]``;
    ``lse`` is the natural-log sum of exp(scaled scores), ``-inf`` for an empty prefix.  The int4
    half of chunked prefill, for which the reference restores the prefix to fp16 first
    (``qslab/runtime/model/attention.py:38-56,119-131``)."""
    total, hq, d = q.shape
    hkv = num_kv_heads if num_kv_heads is not None else hq
    kq, ks = k_cache
    vq, vs = v_cache
    if q.dtype != torch.float16:
        raise TypeError("KV4 attention takes fp16 queries")
    _static_scale(ks, hkv, d)
    if total % rows:
        raise ValueError("the query rows must come in whole blocks")
    out = torch.empty((total, hq, d), dtype=torch.float16, device=q.device)
    lse = torch.empty((total, hq), dtype=torch.float32, device=q.device)
    if total == 0:
        return out, lse
    blocks = total // rows
    if q.stride(2) != 1 or q.stride(1) != d:
        q = q.contiguous()
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    bt = bt if bt.is_contiguous() else bt.contiguous()
    lens = prefix_lens if prefix_lens.dtype == torch.int32 else prefix_lens.to(torch.int32)
    max_blocks = bt.shape[1]
    args = (blocks, rows, hq, hkv, d, block_n, max_blocks)
    with torch.cuda.device(q.device):
        need = _lib.lib.lq2_kv4_attention_workspace_bytes(*args)
        if need == 0:
            raise ValueError(f"unsupported KV4 prefix attention shape: blocks={blocks} rows={rows} HQ={hq} "
                             f"HKV={hkv} D={d} page={block_n} table={max_blocks}")
        ws = _workspace.get("kv4", need, q.device)
        stream = torch.cuda.current_stream().cuda_stream
        status = _lib.lib.lq2_kv4_attention_prefix(
            q.data_ptr(), q.stride(0), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
            bt.data_ptr(), lens.data_ptr(), out.data_ptr(), lse.data_ptr(), blocks, rows, hq, hkv, d, block_n,
            max_blocks, v_group, kq.shape[0], ws.data_ptr(), ws.numel(), stream)
    _lib.check(status, "lq2_kv4_attention_prefix")
    _lib.count()
    return out, lse


def chunk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, first_row: torch.Tensor,
                    prefix_row: torch.Tensor, pre: torch.Tensor | None = None,
                    pre_lse: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of a prefill step's new rows ``q [T, HQ, D]`` over the step's own fp16
    ``k, v [T, HKV, D]`` (row ``i`` sees rows ``first_row[i] .. i``), merged with the prefix part
    ``(pre, pre_lse)`` of ``paged_attention_prefix`` at row ``prefix_row[i]`` (``-1``: no prefix,
    ``-2``: leave ``out[i]`` alone).  Stands in for the flash-attn call of
    ``qslab/runtime/model/attention.py:119-131``."""
    t, hq, d = q.shape
    hkv = k.shape[1]
    if q.dtype != torch.float16 or k.dtype != torch.float16 or v.dtype != torch.float16:
        raise TypeError("chunk attention takes fp16 q, k, v")
    out = torch.empty((t, hq, d), dtype=torch.float16, device=q.device) if out is None else out
    if t == 0:
        return out
    def rows_of(x, heads):
        return x if x.stride(2) == 1 and x.stride(1) == d else x.contiguous()
    q, k, v = rows_of(q, hq), rows_of(k, hkv), rows_of(v, hkv)
    first_row = first_row.to(torch.int32)
    prefix_row = prefix_row.to(torch.int32)
    with torch.cuda.device(q.device):
        status = _lib.lib.lq2_chunk_attention(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), first_row.data_ptr(),
            prefix_row.data_ptr(), pre.data_ptr() if pre is not None else None,
            pre_lse.data_ptr() if pre_lse is not None else None, out.data_ptr(), t, hq, hkv, d,
            torch.cuda.current_stream().cuda_stream)
    _lib.check(status, "lq2_chunk_attention")
    _lib.count()
    return out


def materialize_kv(k_cache, v_cache, slots: torch.Tensor, v_group: int = 64):
    """Dequantise the selected slots to fp16 ``[T, HKV, D]`` (prefix restore,
    ``qslab/kernels/kv4/layout.py:33-47``)."""
    kq, ks = k_cache
    vq, vs = v_cache
    slots = torch.as_tensor(slots, device=kq.device).to(torch.int64).contiguous()
    h, d = kq.shape[1], kq.shape[2] * 8
    _static_scale(ks, h, d)
    t = slots.numel()
    k = torch.empty((t, h, d), dtype=torch.float16, device=kq.device)
    v = torch.empty_like(k)
    if t:
        with torch.cuda.device(kq.device):
            stream = torch.cuda.current_stream().cuda_stream
            status = _lib.lib.lq2_kv4_materialize(
                kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(), slots.data_ptr(),
                k.data_ptr(), v.data_ptr(), t, h, d, v_group, kq.shape[0], stream)
        _lib.check(status, "lq2_kv4_materialize")
        _lib.count()
    return k, v
