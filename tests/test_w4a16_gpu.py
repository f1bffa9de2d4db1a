"""W4A16 kernels on the GPU against the golden fixtures and the CPU oracle.

Packed words are compared bit for bit.  Outputs are compared with the fp32
dequantised reference: max-abs-error / RMS <= 1e-2 (the stated output
tolerance) and relative L2 < 1e-2 (``tests/kernels/test_w4a16.py:57`` of the
reference)."""
import gc

import numpy as np
import pytest
import torch

from oracle import w4a16 as ow

pytestmark = pytest.mark.gpu

TOL = 1e-2
W4_CASES = ["sym_g128", "affine_g128", "affine_g64", "sym_g32"]


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def make_layer(values, scale, zero, group, symmetric, input_scale=None):
    from linkq2_b200.runtime.backends import make_quant_linear
    return make_quant_linear("b200", values, scale, group_size=group, symmetric=symmetric,
                             zero_point=zero, input_scale=input_scale, device="cuda", dtype=torch.float16)


@pytest.mark.parametrize("name", W4_CASES)
def test_golden_pack_and_linear(golden, name):
    g = golden("w4a16")
    n, k, group, affine = (int(v) for v in g[f"{name}.meta"])
    values, scale = t(g[f"{name}.values"]), t(g[f"{name}.scale"])
    zero = t(g[f"{name}.zero_point"]) if affine else None
    layer = make_layer(values, scale, zero, group, not affine)
    assert torch.equal(layer.packed.cpu(), t(g[f"{name}.packed"]))
    assert layer.packed.shape == (k // 8, n) and layer.packed.is_contiguous()
    assert layer.scales.shape == (k // group, n)
    x = t(g[f"{name}.x"]).cuda()
    expected = t(g[f"{name}.y"])
    for rows in (1, 2, 5):
        y = layer(x[:rows]).float().cpu()
        assert ow.error_over_rms(y, expected[:rows]) <= TOL
        assert ow.rel_l2(y, expected[:rows]) < TOL


@pytest.mark.parametrize("affine", [False, True])
@pytest.mark.parametrize("m", [1, 3, 8, 9, 16, 24, 32, 40, 64, 100, 257])
def test_linear_against_oracle_all_row_counts(affine, m):
    n, k, group = 512, 1024, 128
    w = ow.seeded_weight(n, k, seed=11)
    if affine:
        values, scale, zero = ow.affine_quantize(w, group)
    else:
        (values, scale), zero = ow.rtn_quantize(w, group), None
    layer = make_layer(values, scale, zero, group, not affine)
    x = ow.seeded_activation(m, k, seed=100 + m, outliers=True)
    dense = ow.dequantize_fp32(values, scale, symmetric=not affine, zero_point=zero)
    expected = ow.linear_fp32(x, dense)
    y = layer(x.cuda()).float().cpu()
    assert y.shape == (m, n)
    assert ow.error_over_rms(y, expected) <= TOL
    assert ow.rel_l2(y, expected) < TOL


@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 6144), (12288, 4096)])
@pytest.mark.parametrize("affine", [False, True])
def test_projection_shapes_decode_and_batch(k, n, affine):
    """Qwen3-8B projection shapes at M = 1 and M = 16 (full size, compared
    against an fp32 matmul of the oracle's dequantised weight)."""
    w = ow.seeded_weight(n, k, seed=5)
    if affine:
        values, scale, zero = ow.affine_quantize(w, 128)
    else:
        (values, scale), zero = ow.rtn_quantize(w, 128), None
    layer = make_layer(values, scale, zero, 128, not affine)
    packed, _, _ = ow.runtime_buffers(values, scale, symmetric=not affine, zero_point=zero)
    assert torch.equal(layer.packed.cpu(), packed)
    dense = ow.dequantize_fp32(values, scale, symmetric=not affine, zero_point=zero)
    for m in (1, 16):
        x = ow.seeded_activation(m, k, seed=m, outliers=True)
        y = layer(x.cuda()).float().cpu()
        expected = ow.linear_fp32(x, dense)
        assert ow.error_over_rms(y, expected) <= TOL
        assert ow.rel_l2(y, expected) < TOL


@pytest.mark.parametrize("k,n", [(4096, 768), (512, 4096), (4096, 3072), (1536, 4096),      # Qwen3-8B at TP = 8
                                 (4096, 1536), (1024, 4096), (4096, 6144), (3072, 4096),     # TP = 4
                                 (2048, 4096), (4096, 12288), (6144, 4096)])                 # TP = 2
def test_tensor_parallel_shard_shapes(k, n):
    """Per-rank projection shapes of Qwen3-8B under tensor parallelism 2, 4 and 8 (fused
    qkv / gate_up columns, row-split o / down) at M = 1, 32 and 512."""
    w = ow.seeded_weight(n, k, seed=k + n)
    values, scale = ow.rtn_quantize(w, 128)
    layer = make_layer(values, scale, None, 128, True)
    dense = ow.dequantize_fp32(values, scale, symmetric=True)
    for m in (1, 32, 512):
        x = ow.seeded_activation(m, k, seed=m, outliers=True)
        y = layer(x.cuda()).float().cpu()
        expected = ow.linear_fp32(x, dense)
        assert ow.error_over_rms(y, expected) <= TOL
        assert ow.rel_l2(y, expected) < TOL


def test_linearity_and_determinism():
    """Size-independent properties: the op is linear in x up to fp16 rounding
    of the output, and repeated calls return identical bits (split-K partials
    are merged in a fixed order)."""
    n, k = 4096, 4096
    values, scale = ow.rtn_quantize(ow.seeded_weight(n, k, 3), 128)
    layer = make_layer(values, scale, None, 128, True)
    x1 = ow.seeded_activation(1, k, 1).cuda()
    x2 = ow.seeded_activation(1, k, 2).cuda()
    y1, y2, y12 = layer(x1).float(), layer(x2).float(), layer(x1 + x2).float()
    rms = y12.pow(2).mean().sqrt()
    assert ((y1 + y2) - y12).abs().max() / rms < 5e-3
    again = [layer(x1) for _ in range(5)]
    assert all(torch.equal(again[0], a) for a in again)


def test_strided_rows_group_sizes_and_awq_scale():
    n, k = 256, 512
    w = ow.seeded_weight(n, k, 9)
    for group in (32, 64, 256, 512):
        values, scale, zero = ow.affine_quantize(w, group)
        layer = make_layer(values, scale, zero, group, False)
        big = ow.seeded_activation(6, 2 * k, 4).cuda()
        x = big[:, :k]                       # row stride 2K
        assert not x.is_contiguous()
        dense = ow.dequantize_fp32(values, scale, symmetric=False, zero_point=zero)
        expected = ow.linear_fp32(x.cpu(), dense)
        assert ow.error_over_rms(layer(x).float().cpu(), expected) <= TOL
    # AWQ input_scale divides the activations in fp16 first (gemlite.py:41-42)
    values, scale, zero = ow.affine_quantize(w, 128)
    g = torch.Generator().manual_seed(2)
    input_scale = (torch.rand(k, generator=g) + 0.5).half()
    layer = make_layer(values, scale, zero, 128, False, input_scale=input_scale)
    x = ow.seeded_activation(3, k, 8)
    dense = ow.dequantize_fp32(values, scale, symmetric=False, zero_point=zero)
    expected = ow.linear_fp32(x / input_scale, dense)
    assert ow.error_over_rms(layer(x.cuda()).float().cpu(), expected) <= TOL
    # leading dimensions are kept
    y = layer(x.cuda().reshape(3, 1, k))
    assert y.shape == (3, 1, n)


def test_rejects_what_the_reference_rejects():
    values, scale = ow.rtn_quantize(ow.seeded_weight(64, 256, 1), 128)
    with pytest.raises(TypeError):
        make_layer(values, scale, None, 128, True).forward(torch.zeros(1, 256, device="cuda"))
    with pytest.raises(ValueError):
        make_layer(values[:48], scale[:48], None, 128, True)          # N % 32
    with pytest.raises(ValueError):
        make_layer(values, scale, None, 96, True)                       # group not a power of two
    from linkq2_b200.runtime.backends import make_quant_linear
    with pytest.raises(ValueError):
        make_quant_linear("nope", values, scale, group_size=128, symmetric=True, device="cuda",
                          dtype=torch.float16)


def test_buffers_move_and_release():
    """``tests/kernels/test_w4a16.py:59-66`` of the reference: buffers survive
    ``.cpu().cuda()`` and deleting the layer returns memory to the baseline."""
    torch.cuda.synchronize()
    values, scale = ow.rtn_quantize(ow.seeded_weight(256, 1024, 1), 128)
    x = ow.seeded_activation(4, 1024, 3).cuda()
    make_layer(values, scale, None, 128, True)(x)      # creates the cached workspace
    gc.collect()
    torch.cuda.synchronize()
    baseline = torch.cuda.memory_allocated()
    layer = make_layer(values, scale, None, 128, True)
    assert not list(layer.parameters())
    assert layer.weight_memory_bytes() < values.numel()
    before = layer(x)
    layer.cpu().cuda()
    assert all(b.device.type == "cuda" for b in layer.buffers())
    assert torch.equal(layer(x), before)
    del layer, before
    gc.collect()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == baseline


@pytest.mark.parametrize("affine", [False, True])
@pytest.mark.parametrize("k,n", [(256, 128), (4096, 12288), (4096, 1536), (1024, 6144)])
def test_gate_up_with_silu_epilogue_is_bit_identical(k, n, affine):
    """``fuse_gate_up`` (columns interleaved in blocks of four, activation in the kernel's
    epilogue) returns the bits of ``silu_mul`` applied to the plainly concatenated projection
    (same shape, hence the same K split and summation order) for every routed kernel:
    weight-streaming (M <= 8), tcgen05 with pushed reduction (M <= 64) and with pulled
    (M > 64); against the two separate projections, whose K split may differ, it agrees to
    fp16 rounding of the sums."""
    from linkq2_b200.kernels.fused import silu_mul
    from linkq2_b200.runtime.backends.b200 import B200Linear
    layers = []
    for seed in (11, 12):
        w = ow.seeded_weight(n, k, seed=seed + n)
        if affine:
            values, scale, zero = ow.affine_quantize(w, 128)
        else:
            (values, scale), zero = ow.rtn_quantize(w, 128), None
        layers.append(make_layer(values, scale, zero, 128, not affine))
    gate, up = layers
    fused = B200Linear.fuse_gate_up(gate, up)
    plain = B200Linear.fuse_columns([gate, up])
    assert fused.out_features == n and fused.packed.shape == (k // 8, 2 * n)
    for m in (1, 5, 8, 9, 32, 64, 65, 200):
        x = ow.seeded_activation(m, k, seed=m, outliers=True).cuda()
        got = fused(x)
        assert got.shape == (m, n)
        want = silu_mul(*plain(x).chunk(2, dim=-1))
        assert torch.equal(got, want), (m, (got.float() - want.float()).abs().max().item())
        apart = silu_mul(gate(x), up(x)).float()
        assert ((got.float() - apart).abs() <= 4e-3 * apart.abs() + 1e-3).all()
