"""W4A16 Linear backed by the sm_100a kernels of this package.

Drop-in for ``GemLiteLinear`` (``qslab/runtime/backends/gemlite.py:8-43``): same
constructor contract, same buffer names, shapes and dtypes (``packed [K/8, N]
int32``, ``scales [K/G, N] fp16``, ``zeros`` 0-dim int32 8 or ``[K/G, N] fp16``,
``input_scale [K]`` or ``None``), same exceptions - with one gap: the reference's
constructor also takes bf16 activations (``gemlite.py:14``), these kernels compute in fp16
only, as the reference's runtime does (``model_runner.py:33``), and bf16 raises ``TypeError``."""
import torch

from linkq2_b200.kernels.gemlite.bitpack import pack_w4
from linkq2_b200.kernels.gemlite.ops import linear
from linkq2_b200.runtime.backends.base import QuantLinear

# The metadata tuple the reference hands to its kernels (gemlite.py:33-34):
# W_nbits, group_size, unpack_mask, elements_per_sample, input dtype, output
# dtype, accumulator dtype, meta dtype, channel_scale_mode, W_group_mode,
# data_contiguous, type_id.  Dtype codes follow kernels/gemlite/dtypes.py:5-8.
_FP32, _FP16 = 0, 1


def _weights_complete(device):
    """Load-time barrier: the kernels that built the buffers have finished before the
    layer can be called.  With constant weights declared (``set_constant_weights``) the
    linear kernels fetch weight bytes ahead of stream order, so a layer must never be
    called while the kernels that wrote its buffers may still be running."""
    torch.cuda.current_stream(device).synchronize()


class B200Linear(QuantLinear):
    @classmethod
    @torch.no_grad()
    def from_quantized(cls, values, scale, *, group_size, symmetric,
                       zero_point=None, input_scale=None, device, dtype):
        if dtype not in (torch.float16, torch.bfloat16):
            raise TypeError("W4A16 requires FP16 or BF16 activations")
        if dtype != torch.float16:
            raise TypeError("the B200 W4A16 kernels compute in FP16; BF16 activations are not supported")
        n, k = values.shape
        if group_size < 32 or group_size & (group_size - 1) or k % group_size or n % 32:
            raise ValueError(f"unsupported W4A16 shape/group: N={n}, K={k}, group={group_size}")
        if not symmetric and zero_point is None:
            raise ValueError("affine checkpoints need a zero_point tensor")
        layer = cls()
        layer.in_features, layer.out_features = k, n
        layer.group_size, layer.compute_dtype = group_size, dtype
        codes = values.to(device=device)
        codes = codes.to(torch.int8) if codes.dtype not in (torch.int8, torch.uint8) else codes
        layer.register_buffer("packed", pack_w4(codes, symmetric))
        layer.register_buffer("scales", scale.to(device=device, dtype=torch.float16).t().contiguous())
        zeros = (torch.tensor(8, dtype=torch.int32, device=device) if symmetric
                 else zero_point.to(device=device, dtype=torch.float16).t().contiguous())
        layer.register_buffer("zeros", zeros)
        layer.register_buffer("input_scale", None if input_scale is None
                              else input_scale.to(device=device, dtype=dtype))
        layer._meta = (4, group_size, 15, 8, _FP16, _FP16, _FP32, _FP16, 0, 3, True, 104)
        _weights_complete(layer.packed.device)
        return layer

    @classmethod
    @torch.no_grad()
    def fuse_columns(cls, layers):
        """One layer computing ``cat([l(x) for l in layers], -1)``: the packed
        words, scales and zero points of projections that share their input are
        concatenated along N, which the ``[K/8, N]`` layout allows without
        repacking.  Only for layers without an AWQ ``input_scale`` (each AWQ module
        divides its input by its own vector, ``gemlite.py:41-42``) and with equal
        K, group size and zero mode."""
        first = layers[0]
        for l in layers:
            if l.input_scale is not None:
                raise ValueError("projections with an input_scale cannot be fused")
            if (l.in_features, l.group_size, l.zeros.numel() == 1) != \
                    (first.in_features, first.group_size, first.zeros.numel() == 1):
                raise ValueError("projections differ in K, group size or zero mode")
        fused = cls()
        fused.in_features = first.in_features
        fused.out_features = sum(l.out_features for l in layers)
        fused.group_size, fused.compute_dtype = first.group_size, first.compute_dtype
        fused.register_buffer("packed", torch.cat([l.packed for l in layers], dim=1).contiguous())
        fused.register_buffer("scales", torch.cat([l.scales for l in layers], dim=1).contiguous())
        fused.register_buffer("zeros", first.zeros.clone() if first.zeros.numel() == 1
                              else torch.cat([l.zeros for l in layers], dim=1).contiguous())
        fused.register_buffer("input_scale", None)
        fused._meta = first._meta
        _weights_complete(fused.packed.device)
        return fused

    @classmethod
    @torch.no_grad()
    def fuse_gate_up(cls, gate, up):
        """One layer computing ``silu(gate(x)) * up(x)`` in a single launch: the columns of
        the two projections are interleaved in blocks of four, ``[g0..g3 | u0..u3 | g4..``,
        so that every output tile of the kernel holds matching gate and up channels and its
        epilogue can apply the activation (``lq2_w4a16_gate_up_silu``).  Same conditions as
        ``fuse_columns``; ``out_features`` is the intermediate size."""
        fused = cls.fuse_columns([gate, up])
        n = gate.out_features
        if up.out_features != n or n % 32:
            raise ValueError("gate and up projections must have the same width, a multiple of 32")

        def interleave(a, b):
            rows = a.shape[0]
            return torch.stack([a.view(rows, n // 4, 4), b.view(rows, n // 4, 4)], dim=2).reshape(rows, 2 * n)
        fused.packed = interleave(gate.packed, up.packed).contiguous()
        fused.scales = interleave(gate.scales, up.scales).contiguous()
        if gate.zeros.numel() > 1:
            fused.zeros = interleave(gate.zeros, up.zeros).contiguous()
        fused.out_features = n
        fused.gate_up_silu = True
        _weights_complete(fused.packed.device)
        return fused

    def forward_push(self, x, exchange):
        """``forward`` of a row-split projection that also sends the partial sum to the
        tensor-parallel peers (see ``ops.linear``)."""
        if x.dtype != self.compute_dtype:
            raise TypeError(f"expected {self.compute_dtype}, got {x.dtype}")
        return linear(x, self.packed, self.scales, self.zeros, self._meta, push_to=exchange)

    def forward(self, x):
        if getattr(self, "gate_up_silu", False):
            if x.dtype != self.compute_dtype:
                raise TypeError(f"expected {self.compute_dtype}, got {x.dtype}")
            return linear(x, self.packed, self.scales, self.zeros, self._meta, gate_up_silu=True)
        if x.dtype != self.compute_dtype:
            raise TypeError(f"expected {self.compute_dtype}, got {x.dtype}")
        if self.input_scale is not None:
            x = x / self.input_scale
        return linear(x, self.packed, self.scales, self.zeros, self._meta)
