"""CPU oracle for the KV4 cache operators (test infrastructure, never shipped).

Restates with torch CPU tensors:

* ``store_kv_quant`` — ``qslab/kernels/kv4/store.py:9-68``;
* ``paged_attention_decode`` for one query position and for the multi-position
  verify — ``qslab/kernels/kv4/paged_attention.py:11-150`` and
  ``qslab/kernels/kv4/grouped_attention.py:7-63``;
* ``materialize_kv`` — ``qslab/kernels/kv4/layout.py:9-47``;
* ``paged_attention_prefix`` — the pool half of chunked prefill, which the
  reference composes from ``materialize_kv`` and flash-attn
  (``qslab/runtime/model/attention.py:38-56,119-131``).

Pool layout (``qslab/runtime/execute/model_runner.py:146-156``):
``kq, vq [S, HKV, D/8]`` 32-bit words, ``ks [HKV, D] fp16`` static per-channel
table, ``vs [S, HKV, D/v_group] fp16``.  The reference kernels also carry a
dynamic-K branch (one scale per token and head, ``store.py:35-36,42-43``) that
the runtime never configures and that cannot be reached: it is selected by
``ks.dim() != 2`` (``store.py:67``) while the only dynamic pool the reference
builds is two-dimensional (``tests/kernels/test_kv4_paged.py:19``), and the
branch itself fails to trace (``scale[:, 0]`` at ``store.py:43``).  Only the
static table is restated here; any other ``ks`` raises.
Word ``w`` of a head packs channels ``8w .. 8w+7``, channel ``8w+r`` in bits
``4r .. 4r+3`` as the offset-binary nibble ``(code + 8) & 15``.
"""
from __future__ import annotations

import torch


def _words_i64(words: torch.Tensor) -> torch.Tensor:
    """32-bit pool words (uint32 or int32 storage) as non-negative int64."""
    if words.dtype == torch.uint32:
        words = words.view(torch.int32)
    return words.to(torch.int64) & 0xFFFFFFFF


def _store_words(dst: torch.Tensor, index: torch.Tensor, words_i64: torch.Tensor) -> None:
    signed = torch.where(words_i64 >= 2 ** 31, words_i64 - 2 ** 32, words_i64).to(torch.int32)
    view = dst.view(torch.int32) if dst.dtype == torch.uint32 else dst
    view[index] = signed


def _require_static(ks: torch.Tensor, h: int, d: int) -> None:
    if tuple(ks.shape) != (h, d):
        raise ValueError(f"K scale must be the static [HKV, D] = [{h}, {d}] table, got {tuple(ks.shape)}")


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """``[..., D]`` integer codes in -8..7 -> ``[..., D/8]`` int64 words
    (``store.py:38-41``)."""
    nib = (codes.to(torch.int64) + 8) & 0xF
    nib = nib.reshape(*codes.shape[:-1], codes.shape[-1] // 8, 8)
    shifts = torch.arange(8, dtype=torch.int64) * 4
    return (nib << shifts).sum(-1)


def unpack_nibbles(words: torch.Tensor) -> torch.Tensor:
    """``[..., NW]`` pool words -> ``[..., NW*8]`` signed codes -8..7 (int64)."""
    w = _words_i64(words)
    shifts = torch.arange(8, dtype=torch.int64) * 4
    return (((w.unsqueeze(-1) >> shifts) & 0xF) - 8).flatten(-2)


def quantize_codes(x32: torch.Tensor, scale32: torch.Tensor) -> torch.Tensor:
    """``floor(clip(x / s, -8, 7) + 0.5)`` in fp32 with IEEE division
    (``store.py:37`` and ``:49``): clip first, then add one half and floor, so
    ties go up and -8.5.. saturates to -8."""
    return torch.floor(torch.clamp(x32 / scale32, -8.0, 7.0) + 0.5).to(torch.int64)


def store_kv_quant(k, v, k_cache, v_cache, slot_mapping, v_group: int = 64) -> None:
    """Quantize ``k, v [T, HKV, D] fp16`` and scatter them into the pool at
    ``slot_mapping [T]``; ``-1`` skips the token (``store.py:19-22``).

    K: static table ``ks [HKV, D]`` (``store.py:33-34,37``).
    V: per (token, head, group of ``v_group`` channels)
    ``s = max(amax / 7, 1e-4)`` in fp32, codes from the fp32 ``s``, pool keeps
    ``fp16(s)`` (``:46-55``).
    """
    kq, ks = k_cache
    vq, vs = v_cache
    t, h, d = k.shape
    slots = slot_mapping.to(torch.int64)
    keep = slots != -1
    idx = slots[keep]
    k32 = k.float()[keep]
    v32 = v.float()[keep]
    _require_static(ks, h, d)
    k_scale = ks.float().unsqueeze(0)
    # Later tokens overwrite earlier ones when a slot repeats, as a sequential
    # scatter would; index assignment keeps the last write for CPU tensors.
    _store_words(kq, idx, pack_nibbles(quantize_codes(k32, k_scale)))
    vg = v32.reshape(-1, h, d // v_group, v_group)
    v_scale = torch.clamp(vg.abs().amax(-1) / 7.0, min=1e-4)           # [T, H, NG] fp32
    codes = quantize_codes(vg, v_scale.unsqueeze(-1)).reshape(-1, h, d)
    _store_words(vq, idx, pack_nibbles(codes))
    vs[idx] = v_scale.to(torch.float16)


def dequantize_slots(k_cache, v_cache, slots, v_group: int = 64):
    """fp32 ``K, V [T, HKV, D]`` for the given slots:
    ``fp32(nibble - 8) * fp32(scale)`` (``layout.py:22-31``,
    ``paged_attention.py:54-61,74-81``)."""
    kq, ks = k_cache
    vq, vs = v_cache
    slots = torch.as_tensor(slots).to(torch.int64)
    h, d = kq.shape[1], kq.shape[2] * 8
    kc = unpack_nibbles(kq.view(torch.int32)[slots] if kq.dtype == torch.uint32 else kq[slots]).float()
    vc = unpack_nibbles(vq.view(torch.int32)[slots] if vq.dtype == torch.uint32 else vq[slots]).float()
    _require_static(ks, h, d)
    k = kc * ks.float().unsqueeze(0)
    v = (vc.reshape(-1, h, d // v_group, v_group) * vs[slots].float().unsqueeze(-1)).reshape(-1, h, d)
    return k, v


def materialize_kv(k_cache, v_cache, slots, v_group: int = 64):
    """Prefix restore: gather + dequantise to fp16 ``[T, HKV, D]``, order of
    ``slots`` kept, duplicates allowed (``layout.py:33-47``).  The fp32 product
    is rounded once to fp16 by the store at ``layout.py:30-31``."""
    k, v = dequantize_slots(k_cache, v_cache, slots, v_group)
    return k.to(torch.float16), v.to(torch.float16)


def paged_attention_decode(q, k_cache, v_cache, block_tables, context_lens,
                           block_n: int = 128, num_kv_heads: int | None = None,
                           k_scale=None, v_group: int = 64, verify_m: int = 1, out_dtype=torch.float16):
    """``q [rows, HQ, D] fp16 -> out [rows, HQ, D] fp16`` with ``rows = B * M``.

    Row ``seq*M + m`` reads logical positions ``[0, L_seq + m)`` capped at the
    block table's capacity (``paged_attention.py:26-30``); a position whose
    block-table entry is negative is masked (``:49,64``;
    ``grouped_attention.py:38,46``).  Scores are scaled by ``D**-0.5``
    (``:146``), softmax and the value sum are fp32 and a row with no valid key
    yields zeros (``:66-70,84-85``: ``acc / max(l, 1e-20)`` with ``acc = 0``).
    The fp32 result is rounded to fp16 once (``out_dtype=torch.float32`` returns it
    unrounded: the fp32 reference of the output tolerance).
    """
    rows, hq, d = q.shape
    hkv = num_kv_heads if num_kv_heads is not None else hq
    rep = hq // hkv
    m_rows = verify_m
    batch = rows // m_rows
    page = block_n
    capacity = block_tables.shape[1] * page
    out = torch.zeros(rows, hq, d, dtype=torch.float32)
    heads = torch.arange(hq) // rep
    bt = block_tables.to(torch.int64)
    for seq in range(batch):
        length = int(context_lens[seq])
        hi = min(length + m_rows - 1, capacity)
        if hi <= 0:
            continue
        pos = torch.arange(hi)
        raw = bt[seq, pos // page]
        slots = torch.clamp(raw, min=0) * page + pos % page
        k, v = dequantize_slots(k_cache, v_cache, slots, v_group)       # [hi, HKV, D]
        kh = k[:, heads].permute(1, 0, 2)                               # [HQ, hi, D]
        vh = v[:, heads].permute(1, 0, 2)
        for m in range(m_rows):
            row = seq * m_rows + m
            valid = (pos < min(length + m, capacity)) & (raw >= 0)
            if not bool(valid.any()):
                continue
            scores = torch.einsum("hd,htd->ht", q[row].float(), kh) * (d ** -0.5)
            scores = scores.masked_fill(~valid.unsqueeze(0), float("-inf"))
            out[row] = torch.einsum("ht,htd->hd", torch.softmax(scores, -1), vh)
    return out.to(out_dtype)


def paged_attention_prefix(q, k_cache, v_cache, block_tables, prefix_lens, block_n: int = 128,
                           num_kv_heads: int | None = None, v_group: int = 64, rows: int = 16):
    """The pool half of chunked-prefill attention: every row of block ``b`` (``rows`` rows of
    ``q [blocks*rows, HQ, D]``) attends to the dequantised positions ``[0, prefix_lens[b])`` of
    ``block_tables[b]``.  Returns fp32 ``(out, lse)``, ``lse`` the natural-log sum of
    exp(scaled scores), ``-inf`` and zeros for an empty prefix.  The reference gets the same
    numbers by restoring the prefix with ``materialize_kv`` and handing it to flash-attn in
    front of the step's own rows (``qslab/runtime/model/attention.py:38-56,119-131``)."""
    total, hq, d = q.shape
    hkv = num_kv_heads if num_kv_heads is not None else hq
    heads = torch.arange(hq) // (hq // hkv)
    out = torch.zeros(total, hq, d, dtype=torch.float32)
    lse = torch.full((total, hq), float("-inf"), dtype=torch.float32)
    bt = block_tables.to(torch.int64)
    for b in range(total // rows):
        n = min(int(prefix_lens[b]), block_tables.shape[1] * block_n)
        if n <= 0:
            continue
        pos = torch.arange(n)
        raw = bt[b, pos // block_n]
        keep = raw >= 0
        if not bool(keep.any()):
            continue
        slots = (raw * block_n + pos % block_n)[keep]
        k, v = dequantize_slots(k_cache, v_cache, slots, v_group)
        qb = q[b * rows:(b + 1) * rows].float()
        scores = torch.einsum("rhd,thd->rht", qb, k[:, heads]) * (d ** -0.5)
        part = torch.logsumexp(scores, dim=-1)
        lse[b * rows:(b + 1) * rows] = part
        out[b * rows:(b + 1) * rows] = torch.einsum("rht,thd->rhd", torch.exp(scores - part.unsqueeze(-1)), v[:, heads])
    return out, lse


def chunk_attention(q, k, v, first_row, prefix_row, pre=None, pre_lse=None):
    """Causal attention of a step's new rows over the step's own fp16 ``k, v`` (row ``i`` sees
    rows ``first_row[i] .. i``), merged with the prefix part ``pre[prefix_row[i]]`` weighted by
    ``exp(pre_lse)`` against the own part's sum of exponentials; fp32 ``[T, HQ, D]``, rows with
    ``prefix_row == -2`` left at zero.  Together with ``paged_attention_prefix`` this is the
    softmax over prefix + own keys that the reference computes in one flash-attn call
    (``qslab/runtime/model/attention.py:119-131``)."""
    t, hq, d = q.shape
    heads = torch.arange(hq) // (hq // k.shape[1])
    out = torch.zeros(t, hq, d, dtype=torch.float32)
    for i in range(t):
        pr = int(prefix_row[i])
        if pr < -1:
            continue
        f = int(first_row[i])
        kk, vv = k[f:i + 1].float()[:, heads], v[f:i + 1].float()[:, heads]        # [n, HQ, D]
        s = torch.einsum("hd,nhd->hn", q[i].float(), kk) * (d ** -0.5)
        own_lse = torch.logsumexp(s, dim=-1)
        own = torch.einsum("hn,nhd->hd", torch.exp(s - own_lse.unsqueeze(-1)), vv)
        if pr >= 0:
            w = torch.sigmoid(pre_lse[pr].float() - own_lse).unsqueeze(-1)          # the prefix part's share
            own = own + (pre[pr].float() - own) * w
        out[i] = own
    return out


# --------------------------------------------------------------------------
# seeded inputs of the benchmark configuration
# --------------------------------------------------------------------------
def seeded_kv(tokens: int, hkv: int, d: int, seed: int, outlier_channels: int = 4):
    """``K, V [T, HKV, D] fp16 ~ N(0,1)`` with ``outlier_channels`` seeded
    channels per head multiplied by 10."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(tokens, hkv, d, generator=g)
    v = torch.randn(tokens, hkv, d, generator=g)
    for h in range(hkv):
        ck = torch.randperm(d, generator=g)[:outlier_channels]
        cv = torch.randperm(d, generator=g)[:outlier_channels]
        k[:, h, ck] *= 10
        v[:, h, cv] *= 10
    return k.to(torch.float16), v.to(torch.float16)


def static_k_scale(k: torch.Tensor) -> torch.Tensor:
    """Per (head, channel) table ``max(amax_t |K|, 1e-4) / 7`` cast to fp16: the
    rule of ``scripts/build_smooth_kv.py:89`` with lambda = 1."""
    return (k.float().abs().amax(0).clamp_min(1e-4) / 7).to(torch.float16)


def empty_pool(slots: int, hkv: int, d: int, v_group: int = 64, word_dtype=torch.int32):
    """Zeroed pool tensors shaped as ``model_runner.py:146-156`` allocates them."""
    kq = torch.zeros(slots, hkv, d // 8, dtype=word_dtype)
    vq = torch.zeros(slots, hkv, d // 8, dtype=word_dtype)
    ks = torch.zeros(hkv, d, dtype=torch.float16)
    vs = torch.zeros(slots, hkv, d // v_group, dtype=torch.float16)
    return (kq, ks), (vq, vs)
