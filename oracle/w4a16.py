"""CPU oracle for the W4A16 linear path (test infrastructure, never shipped).

Restates, with torch CPU tensors:

* the two weight quantizers that produce checkpoint tensors
  (``qslab/compression/algorithms/rtn.py:15-29``,
  ``qslab/compression/algorithms/awq_affine.py:33-38`` with a unit activation
  statistic, which is how ``tests/kernels/test_w4a16.py:32-33`` obtains an
  asymmetric tensor without calibration data);
* the load-time buffer construction of ``GemLiteLinear.from_quantized``
  (``qslab/runtime/backends/gemlite.py:10-35``) including the int32 packing of
  ``pack_weights_over_cols_triton`` (``qslab/kernels/gemlite/bitpack.py:63-125``);
* the fp32 dequantised reference ``RuntimeQuantization.dequantize``
  (``qslab/runtime/quantization_strategies.py:15-20``, AWQ variant ``:41-42``)
  followed by an fp32 matmul — the quantity ``tests/kernels/test_w4a16.py:51-58``
  compares the GPU kernels against.
"""
from __future__ import annotations

import torch


# --------------------------------------------------------------------------
# quantizers (checkpoint producers)
# --------------------------------------------------------------------------
def rtn_quantize(weight: torch.Tensor, group_size: int = 128, clip_ratio: float = 1.0):
    """Symmetric round-to-nearest W4 (``compression/algorithms/rtn.py:15-29``).

    Returns ``values int8 [N,K]`` in -8..7, ``scale fp16 [N,K/G]``.
    """
    n, k = weight.shape
    if k % group_size:
        raise ValueError("input width must be divisible by group_size")
    grouped = weight.float().reshape(n, -1, group_size)
    scale = (grouped.abs().amax(-1, keepdim=True) * clip_ratio / 7).clamp_min(1e-12)
    values = torch.round(grouped / scale).clamp(-8, 7).to(torch.int8)
    return values.reshape(n, k).contiguous(), scale.squeeze(-1).to(torch.float16)


def affine_quantize(weight: torch.Tensor, group_size: int = 128):
    """Asymmetric uint4 with a per-group zero point.

    This is the grid step of ``compression/algorithms/awq_affine.py:33-38`` for a
    unit activation statistic: with ``activation_absmean == 1`` every candidate
    of the search (``:28-31``) is the all-ones vector, so the search returns the
    plain affine quantization and an all-ones ``input_scale``.

    Returns ``values uint8 [N,K]`` in 0..15, ``scale fp16 [N,K/G]``,
    ``zero_point fp16 [N,K/G]`` (integer valued).
    """
    n, k = weight.shape
    if k % group_size:
        raise ValueError("input width must be divisible by group_size")
    grouped = weight.float().reshape(n, -1, group_size)
    lo = grouped.amin(-1, keepdim=True)
    hi = grouped.amax(-1, keepdim=True)
    scale = ((hi - lo) / 15).clamp_min(1e-12)
    zero = torch.round(-lo / scale).clamp(0, 15)
    values = torch.round(grouped / scale + zero).clamp(0, 15).to(torch.uint8)
    return (values.reshape(n, k).contiguous(), scale.squeeze(-1).to(torch.float16),
            zero.squeeze(-1).to(torch.float16))


# --------------------------------------------------------------------------
# load-time buffers
# --------------------------------------------------------------------------
def codes_from_values(values: torch.Tensor, symmetric: bool) -> torch.Tensor:
    """Unsigned 4-bit codes (``runtime/backends/gemlite.py:22-23``): symmetric
    checkpoints store -8..7 and are offset by +8, affine ones store 0..15."""
    codes = values.to(torch.int16)
    return (codes + 8 if symmetric else codes).to(torch.uint8)


def pack_w4(codes: torch.Tensor) -> torch.Tensor:
    """``[N,K] uint8`` codes -> ``[K/8,N] int32`` contiguous.

    ``word[k8, n] = sum_j codes[n, 8*k8 + j] << (4*j)``: the reduction of
    ``pack_weights_over_cols_kernel`` (``kernels/gemlite/bitpack.py:76-93``)
    followed by the transpose of ``:123`` and the ``.contiguous()`` of
    ``runtime/backends/gemlite.py:25``.
    """
    n, k = codes.shape
    if k % 8:
        raise ValueError("K must be a multiple of 8")
    c = codes.to(torch.int64).reshape(n, k // 8, 8)
    shifts = torch.arange(8, dtype=torch.int64) * 4
    words = (c << shifts).sum(-1)                       # 0 .. 2^32-1
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words.t().contiguous()


def unpack_w4(packed: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`pack_w4`: ``[K/8,N] int32`` -> ``[N,K] uint8`` codes."""
    k8, n = packed.shape
    w = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, dtype=torch.int64) * 4
    nib = (w.unsqueeze(-1) >> shifts) & 0xF             # [K/8, N, 8]
    return nib.permute(1, 0, 2).reshape(n, k8 * 8).to(torch.uint8)


def runtime_buffers(values, scale, *, symmetric, zero_point=None):
    """The three device buffers of a W4 layer, on CPU
    (``runtime/backends/gemlite.py:22-29``): ``packed [K/8,N] int32``,
    ``scales [K/G,N] fp16`` and ``zeros`` — a 0-dim int32 tensor holding 8 for
    symmetric checkpoints, else ``[K/G,N] fp16``."""
    packed = pack_w4(codes_from_values(values, symmetric))
    scales = scale.t().contiguous()
    zeros = torch.tensor(8, dtype=torch.int32) if symmetric else zero_point.t().contiguous()
    return packed, scales, zeros


# --------------------------------------------------------------------------
# arithmetic
# --------------------------------------------------------------------------
def dequantize_fp32(values, scale, *, symmetric, zero_point=None, input_scale=None):
    """Dense fp32 ``[N,K]`` weight, ``(values - zero) * scale`` per group
    (``runtime/quantization_strategies.py:15-20``); AWQ checkpoints divide by
    ``input_scale`` (``:41-42``).  ``values`` are the checkpoint's logical
    integers: -8..7 (symmetric, zero 0) or 0..15 (affine, per-group zero)."""
    s = scale.float()
    zero = 0 if symmetric else zero_point.float().unsqueeze(-1)
    dense = ((values.float().reshape(*s.shape, -1) - zero) * s.unsqueeze(-1)).reshape(values.shape)
    if input_scale is not None:
        dense = dense / input_scale.float()
    return dense


def dequantize_buffers_fp32(packed, scales, zeros):
    """fp32 ``[N,K]`` weight from the *runtime* buffers: ``(u - z) * s`` with
    ``u`` the unsigned code (``kernels/gemlite/triton_kernels/utils.py:66-71``
    evaluated in fp32 instead of fp16)."""
    codes = unpack_w4(packed).float()                   # [N, K]
    n, k = codes.shape
    groups = scales.shape[0]
    s = scales.float().t().unsqueeze(-1)                # [N, G, 1]
    z = (zeros.float().reshape(1, 1, 1) if zeros.numel() == 1
         else zeros.float().t().unsqueeze(-1))
    return ((codes.reshape(n, groups, -1) - z) * s).reshape(n, k)


def linear_fp32(x: torch.Tensor, dense_fp32: torch.Tensor) -> torch.Tensor:
    """``x.float() @ dense.T`` — the expected value of
    ``tests/kernels/test_w4a16.py:55``."""
    return x.float() @ dense_fp32.t()


def linear(x, packed, scales, zeros, input_scale=None):
    """Whole CPU path of one W4A16 layer call: optional AWQ division in the
    activation dtype (``runtime/backends/gemlite.py:41-42``), fp32 dequant of
    the runtime buffers, fp32 matmul.  This is what the CPU baseline times."""
    if input_scale is not None:
        x = x / input_scale
    lead = x.shape[:-1]
    y = linear_fp32(x.reshape(-1, x.shape[-1]), dequantize_buffers_fp32(packed, scales, zeros))
    return y.reshape(*lead, -1)


def error_over_rms(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """max-abs-error divided by the RMS of the expected output: the figure the
    1e-2 output tolerance is stated in."""
    e = expected.float()
    return float((actual.float() - e).abs().max() / e.pow(2).mean().sqrt().clamp_min(1e-30))


def rel_l2(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """``|a-e| / |e|`` (``tests/kernels/test_w4a16.py:57``)."""
    e = expected.float()
    return float((actual.float() - e).norm() / e.norm().clamp_min(1e-30))


# --------------------------------------------------------------------------
# seeded inputs of the benchmark configurations
# --------------------------------------------------------------------------
def seeded_weight(n: int, k: int, seed: int) -> torch.Tensor:
    """fp16 ``[N,K] ~ N(0, 0.02^2)``."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)


def seeded_activation(m: int, k: int, seed: int, outliers: bool = False) -> torch.Tensor:
    """fp16 ``[M,K] ~ N(0,1)``; with ``outliers`` 1 % of the K columns (seeded
    choice) are multiplied by 20."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    if outliers:
        cols = torch.randperm(k, generator=g)[: max(1, k // 100)]
        x[:, cols] *= 20
    return x.to(torch.float16)
