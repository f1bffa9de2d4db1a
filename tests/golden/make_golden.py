"""Regenerate the golden fixtures in this directory from the LinkQ2 reference.

Run where a checkout of the reference is available (it is not needed to *use*
the fixtures)::

    LINKQ2_REFERENCE=/path/to/LinkQ2 python tests/golden/make_golden.py

The reference's Triton kernels are executed on CPU tensors by the Triton
interpreter (``TRITON_INTERPRET=1``); its quantizers and its fp32 dequantised
``RuntimeQuantization.dequantize`` are plain torch.  Every array written here is
an output of reference code on the seeded inputs stored beside it.  Nothing in
this script calls the oracle or the CUDA kernels.
"""
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

REFERENCE = os.environ.get("LINKQ2_REFERENCE")          # a checkout of chuoer47/LinkQ2
if not REFERENCE:
    raise SystemExit("set LINKQ2_REFERENCE to a checkout of the reference (the directory that holds qslab/)")
sys.path.insert(0, REFERENCE)
OUT = Path(__file__).resolve().parent


def _np(t):
    t = t.detach().cpu()
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.numpy()


def w4a16_cases():
    from qslab.compression.algorithms import AWQAffine, RTN
    from qslab.kernels.gemlite.bitpack import pack_weights_over_cols_triton
    from qslab.runtime.quantization_strategies import AWQAffineRuntime, RTNRuntime

    out = {}
    for name, (n, k, group, affine, seed) in {
        "sym_g128": (64, 512, 128, False, 123),
        "affine_g128": (64, 512, 128, True, 124),
        "affine_g64": (32, 256, 64, True, 125),
        "sym_g32": (96, 128, 32, False, 126),
    }.items():
        g = torch.Generator().manual_seed(seed)
        weight = (torch.randn(n, k, generator=g) * 0.02).half()
        quantizer = AWQAffine() if affine else RTN()
        q, transform = quantizer.quantize(weight.float(), group_size=group,
                                          activation_absmean=torch.ones(k))
        codes = q.values.to(torch.int16)
        codes = (codes if affine else codes + 8).to(torch.uint8)
        packed, _ = pack_weights_over_cols_triton(codes, 4, 32, transpose=True)
        packed = packed.contiguous()
        strategy = AWQAffineRuntime() if affine else RTNRuntime()
        data = {"values": q.values, "scale": q.scale,
                "zero_point": q.zero_point if affine else None, "input_scale": transform}
        dense = strategy.dequantize(data)
        x = torch.randn(5, k, generator=g).half()
        scaled = x if transform is None else x / transform
        y = scaled.float() @ dense.t()
        out.update({
            f"{name}.weight": _np(weight), f"{name}.values": _np(q.values),
            f"{name}.scale": _np(q.scale), f"{name}.zero_point": _np(q.zero_point),
            f"{name}.packed": _np(packed), f"{name}.dense": _np(dense),
            f"{name}.x": _np(x), f"{name}.y": _np(y),
            f"{name}.meta": np.array([n, k, group, int(affine)]),
        })
        if transform is not None:
            out[f"{name}.input_scale"] = _np(transform)
    np.savez_compressed(OUT / "w4a16.npz", **out)
    print("w4a16.npz", len(out), "arrays")


def _pool(slots, h, d, group, static, gen):
    kq = torch.zeros(slots, h, d // 8, dtype=torch.int32)
    vq = torch.zeros(slots, h, d // 8, dtype=torch.int32)
    ks = ((torch.rand(h, d, generator=gen) * 0.3 + 0.1).half() if static
          else torch.zeros(slots, h, 1, dtype=torch.float16))
    vs = torch.zeros(slots, h, d // group, dtype=torch.float16)
    return (kq, ks), (vq, vs)


def kv4_store_cases():
    from qslab.kernels.kv4 import materialize_kv, store_kv_quant
    out = {}
    for name, (t, h, d, group, static, strided, seed) in {
        "static_g64": (12, 8, 128, 64, True, False, 0),
        "static_g32_strided": (19, 8, 128, 32, True, True, 19),
        "static_g128": (9, 2, 128, 128, True, False, 20),
        "static_d64": (11, 4, 64, 64, True, False, 21),
    }.items():
        g = torch.Generator().manual_seed(seed)
        slots_total = 40
        if strided:
            fused = (torch.randn(t, h * 3, d, generator=g) * 2).half()
            _, k, v = fused.chunk(3, dim=1)
        else:
            k = (torch.randn(t, h, d, generator=g) * 2).half()
            v = (torch.randn(t, h, d, generator=g) * 2).half()
        # exact ties and saturation, which the rounding rule is about
        k = k.clone() if not strided else k
        kc, vc = _pool(slots_total, h, d, group, static, g)
        slots = torch.randperm(slots_total, generator=g)[:t].int()
        slots[1] = -1
        store_kv_quant(k, v, kc, vc, slots, v_group=group)
        sel = torch.tensor([int(slots[0]), int(slots[3]), int(slots[0]), int(slots[5]), int(slots[2])])
        km, vm = materialize_kv(kc, vc, sel, v_group=group)
        out.update({
            f"{name}.k": _np(k.contiguous()), f"{name}.v": _np(v.contiguous()),
            f"{name}.slots": _np(slots), f"{name}.kq": _np(kc[0]), f"{name}.ks": _np(kc[1]),
            f"{name}.vq": _np(vc[0]), f"{name}.vs": _np(vc[1]),
            f"{name}.sel": _np(sel), f"{name}.km": _np(km), f"{name}.vm": _np(vm),
            f"{name}.meta": np.array([t, h, d, group, int(static), int(strided), slots_total]),
        })
    # rounding ties: k / ks lands exactly on x.5 and beyond the clip range
    h, d, group = 1, 64, 64
    ks = torch.full((h, d), 0.25, dtype=torch.float16)
    ladder = (torch.arange(d, dtype=torch.float32) - 32) * 0.125        # -4 .. 3.875 => codes -16..15.5
    k = ladder.reshape(1, h, d).half()
    v = ladder.reshape(1, h, d).half()
    kc = (torch.zeros(4, h, d // 8, dtype=torch.int32), ks)
    vc = (torch.zeros(4, h, d // 8, dtype=torch.int32), torch.zeros(4, h, 1, dtype=torch.float16))
    store_kv_quant(k, v, kc, vc, torch.tensor([2], dtype=torch.int32), v_group=group)
    out.update({"ties.k": _np(k), "ties.v": _np(v), "ties.ks": _np(ks), "ties.kq": _np(kc[0]),
                "ties.vq": _np(vc[0]), "ties.vs": _np(vc[1])})
    np.savez_compressed(OUT / "kv4_store.npz", **out)
    print("kv4_store.npz", len(out), "arrays")


def kv4_attention_cases():
    from qslab.kernels.kv4 import paged_attention_decode, store_kv_quant
    out = {}
    cases = {
        # name: (bs, lens, M, hq, hkv, d, page, group, table_width, seed)
        "decode_small": (2, [200, 300], 1, 16, 8, 128, 128, 64, 3, 0),
        "decode_split": (1, [700], 1, 8, 2, 128, 128, 64, 8, 1),
        "verify_small": (3, [130, 77, 5], 5, 4, 2, 64, 32, 64, 8, 2),
        "verify_m16": (1, [300], 16, 8, 2, 128, 128, 64, 4, 3),
        "verify_neg1": (1, [100], 4, 4, 2, 64, 32, 64, 20, 5),
        "decode_g32": (2, [64, 129], 1, 4, 1, 128, 128, 32, 2, 6),
    }
    for name, (bs, lens, m, hq, hkv, d, page, group, width, seed) in cases.items():
        g = torch.Generator().manual_seed(seed)
        blocks_needed = [(l + m + page - 1) // page for l in lens]
        n_blocks = sum(blocks_needed) + 2
        slots_total = n_blocks * page
        k = (torch.randn(slots_total, hkv, d, generator=g) * 0.5).half()
        v = (torch.randn(slots_total, hkv, d, generator=g) * 0.5).half()
        ks = (k.float().abs().amax(0) / 7).clamp_min(1e-4).half()
        kc = (torch.zeros(slots_total, hkv, d // 8, dtype=torch.int32), ks)
        vc = (torch.zeros(slots_total, hkv, d // 8, dtype=torch.int32),
              torch.zeros(slots_total, hkv, d // group, dtype=torch.float16))
        store_kv_quant(k, v, kc, vc, torch.arange(slots_total, dtype=torch.int32), v_group=group)
        perm = torch.randperm(n_blocks, generator=g).tolist()
        table = torch.full((bs, width), -1, dtype=torch.int32)
        for i, nb in enumerate(blocks_needed):
            ids, perm = perm[:nb], perm[nb:]
            if name == "verify_neg1":
                ids = ids[:3]                      # rows run past the real blocks
            table[i, :len(ids)] = torch.tensor(ids, dtype=torch.int32)
        ctx = torch.tensor(lens, dtype=torch.int32)
        q = (torch.randn(bs * m, hq, d, generator=g) * 0.5).half()
        o = paged_attention_decode(q, kc, vc, table, ctx, block_n=page, num_kv_heads=hkv,
                                   v_group=group, verify_m=m)
        out.update({
            f"{name}.kq": _np(kc[0]), f"{name}.ks": _np(ks), f"{name}.vq": _np(vc[0]),
            f"{name}.vs": _np(vc[1]), f"{name}.table": _np(table), f"{name}.lens": _np(ctx),
            f"{name}.q": _np(q), f"{name}.out": _np(o),
            f"{name}.meta": np.array([bs, m, hq, hkv, d, page, group]),
        })
    np.savez_compressed(OUT / "kv4_attention.npz", **out)
    print("kv4_attention.npz", len(out), "arrays")


if __name__ == "__main__":
    torch.manual_seed(0)
    w4a16_cases()
    kv4_store_cases()
    kv4_attention_cases()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size, "bytes")
