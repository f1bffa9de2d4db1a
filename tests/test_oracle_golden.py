"""The CPU oracle against outputs of the reference itself.

The fixtures under ``tests/golden`` were produced by ``make_golden.py`` from the
reference's own code (Triton kernels run by the Triton CPU interpreter,
quantizers and the fp32 dequantised weight in torch).  Integer and byte results
must be identical; attention outputs are compared with the tolerance the
reference's tests use (``tests/kernels/test_kv4_verify.py:116``: 2e-3).
"""
import numpy as np
import pytest
import torch

from oracle import kv4, w4a16

W4_CASES = ["sym_g128", "affine_g128", "affine_g64", "sym_g32"]
STORE_CASES = ["static_g64", "static_g32_strided", "static_g128", "static_d64"]
ATTN_CASES = ["decode_small", "decode_split", "verify_small", "verify_m16", "verify_neg1", "decode_g32"]


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_rtn_known_answer():
    """``tests/compression/test_algorithms.py:15-21`` of the reference."""
    weight = torch.tensor([[-7., -3., 0., 7., -14., -6., 0., 14.]])
    values, scale = w4a16.rtn_quantize(weight, group_size=4)
    assert values.tolist() == [[-7, -3, 0, 7, -7, -3, 0, 7]]
    assert scale.tolist() == [[1., 2.]]
    dense = w4a16.dequantize_fp32(values, scale, symmetric=True)
    assert torch.equal(dense, weight)


@pytest.mark.parametrize("name", W4_CASES)
def test_w4a16_oracle_matches_reference(golden, name):
    g = golden("w4a16")
    n, k, group, affine = (int(v) for v in g[f"{name}.meta"])
    weight = t(g[f"{name}.weight"])
    if affine:
        values, scale, zero = w4a16.affine_quantize(weight, group)
        assert torch.equal(zero, t(g[f"{name}.zero_point"]))
        assert torch.equal(t(g[f"{name}.input_scale"]).float(), torch.ones(k))
    else:
        values, scale = w4a16.rtn_quantize(weight, group)
        zero = None
    assert torch.equal(values.to(torch.int16), t(g[f"{name}.values"]).to(torch.int16))
    assert torch.equal(scale, t(g[f"{name}.scale"]))
    packed, scales, zeros = w4a16.runtime_buffers(values, scale, symmetric=not affine, zero_point=zero)
    assert torch.equal(packed, t(g[f"{name}.packed"]))
    assert packed.shape == (k // 8, n) and packed.is_contiguous()
    assert torch.equal(w4a16.unpack_w4(packed), w4a16.codes_from_values(values, not affine))
    dense = w4a16.dequantize_fp32(values, scale, symmetric=not affine, zero_point=zero)
    assert torch.equal(dense, t(g[f"{name}.dense"]))
    assert torch.equal(w4a16.dequantize_buffers_fp32(packed, scales, zeros), dense)
    x = t(g[f"{name}.x"])
    y = w4a16.linear(x, packed, scales, zeros)
    assert w4a16.error_over_rms(y, t(g[f"{name}.y"])) < 1e-5


@pytest.mark.parametrize("name", STORE_CASES)
def test_kv4_store_and_materialize_bit_exact(golden, name):
    g = golden("kv4_store")
    tokens, h, d, group, static, strided, slots_total = (int(v) for v in g[f"{name}.meta"])
    k, v = t(g[f"{name}.k"]), t(g[f"{name}.v"])
    if strided:      # same values through a fused-QKV style view
        fused = torch.zeros(tokens, h * 3, d, dtype=torch.float16)
        fused[:, h:2 * h], fused[:, 2 * h:] = k, v
        _, k, v = fused.chunk(3, dim=1)
        assert not k.is_contiguous()
    kc, vc = kv4.empty_pool(slots_total, h, d, group)
    kc[1].copy_(t(g[f"{name}.ks"]))
    kv4.store_kv_quant(k, v, kc, vc, t(g[f"{name}.slots"]), v_group=group)
    assert torch.equal(kc[0], t(g[f"{name}.kq"]))
    assert torch.equal(vc[0], t(g[f"{name}.vq"]))
    assert torch.equal(vc[1], t(g[f"{name}.vs"]))
    assert torch.equal(kc[1], t(g[f"{name}.ks"]))
    km, vm = kv4.materialize_kv(kc, vc, t(g[f"{name}.sel"]), v_group=group)
    assert torch.equal(km, t(g[f"{name}.km"]))
    assert torch.equal(vm, t(g[f"{name}.vm"]))


def test_kv4_store_ties_and_saturation(golden):
    g = golden("kv4_store")
    k, v, ks = t(g["ties.k"]), t(g["ties.v"]), t(g["ties.ks"])
    kc = (torch.zeros(4, 1, 8, dtype=torch.int32), ks)
    vc = (torch.zeros(4, 1, 8, dtype=torch.int32), torch.zeros(4, 1, 1, dtype=torch.float16))
    kv4.store_kv_quant(k, v, kc, vc, torch.tensor([2], dtype=torch.int32), v_group=64)
    assert torch.equal(kc[0], t(g["ties.kq"]))
    assert torch.equal(vc[0], t(g["ties.vq"]))
    assert torch.equal(vc[1], t(g["ties.vs"]))
    codes = kv4.unpack_nibbles(kc[0][2, 0])
    assert codes.min() == -8 and codes.max() == 7
    # x.5 goes up: k/ks = -0.5 -> floor(0.0) = 0 ; +0.5 -> 1
    assert int(codes[31]) == 0 and int(codes[33]) == 1


@pytest.mark.parametrize("name", ATTN_CASES)
def test_kv4_attention_matches_reference(golden, name):
    g = golden("kv4_attention")
    bs, m, hq, hkv, d, page, group = (int(v) for v in g[f"{name}.meta"])
    kc = (t(g[f"{name}.kq"]), t(g[f"{name}.ks"]))
    vc = (t(g[f"{name}.vq"]), t(g[f"{name}.vs"]))
    out = kv4.paged_attention_decode(t(g[f"{name}.q"]), kc, vc, t(g[f"{name}.table"]),
                                     t(g[f"{name}.lens"]), block_n=page, num_kv_heads=hkv,
                                     v_group=group, verify_m=m)
    ref = t(g[f"{name}.out"])
    assert torch.isfinite(out).all()
    assert (out.float() - ref.float()).abs().max().item() < 2e-3


# ---------------------------------------------------------------------------
# whole model: oracle.qwen3 against the reference's CPU model path
# ---------------------------------------------------------------------------
MODEL_CASES = ["rtn_tied", "rtn_perm", "affine_perm"]


def golden_model_weights(g, tag):
    """Weights of a golden checkpoint in the form ``OracleQwen3`` takes (dense fp32
    projections as the reference's fake load path builds them, fp16 for the rest) and
    its model config."""
    import json
    from types import SimpleNamespace
    raw = json.loads(bytes(g[f"{tag}.config"]).decode())
    layers = json.loads(bytes(g[f"{tag}.layers"]).decode())
    symmetric = bool(raw["quantization_config"]["symmetric"])
    prefix = f"{tag}.ckpt."
    ckpt = {k[len(prefix):]: t(g[k]) for k in g.files if k.startswith(prefix)}
    weights = {}
    for name in layers:
        key = name + ".weight"
        weights[key] = w4a16.dequantize_fp32(ckpt[key], ckpt[key + ".scale"], symmetric=symmetric,
                                             zero_point=ckpt.get(key + ".zero_point"),
                                             input_scale=ckpt.get(key + ".input_scale"))
    for name, tensor in ckpt.items():
        if name.count(".weight") == 1 and name.endswith(".weight") and name not in weights:
            weights[name] = tensor
    theta = raw.get("rope_theta") or raw["rope_parameters"]["rope_theta"]
    cfg = SimpleNamespace(num_hidden_layers=raw["num_hidden_layers"], num_attention_heads=raw["num_attention_heads"],
                          num_key_value_heads=raw["num_key_value_heads"], head_dim=raw["head_dim"],
                          rms_norm_eps=raw["rms_norm_eps"], rope_theta=theta, vocab_size=raw["vocab_size"])
    return cfg, weights


@pytest.mark.parametrize("tag", MODEL_CASES)
def test_model_oracle_matches_reference_cpu_model(golden, tag):
    """Layer graph, norms, RoPE convention, residual handling and head of
    ``oracle.qwen3`` against HF ``Qwen3ForCausalLM`` on the reference's fake (dense)
    weights.  That model has no cache quantization, so the oracle runs with it
    bypassed; logits within 2e-2 of their RMS (the oracle rounds activations to fp16
    between operators, the golden run is fp32) and identical greedy tokens."""
    from oracle import qwen3 as oq
    g = golden("qwen3_tiny")
    cfg, weights = golden_model_weights(g, tag)
    kscale = torch.full((cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim), 0.3)
    for i in range(2):
        prompt = [int(v) for v in g[f"{tag}.prompt{i}"]]
        want_logits = t(g[f"{tag}.prompt{i}.logits"])
        want_tokens = [int(v) for v in g[f"{tag}.prompt{i}.tokens"]]
        oracle = oq.OracleQwen3(cfg, weights, kscale=kscale, max_tokens=256, kv_mode="fp16")
        logits = oracle.forward(prompt, "prefill")
        err = (logits - want_logits).abs().max() / want_logits.pow(2).mean().sqrt()
        assert err < 2e-2, float(err)
        oracle = oq.OracleQwen3(cfg, weights, kscale=kscale, max_tokens=256, kv_mode="fp16")
        assert oracle.greedy(prompt, len(want_tokens)) == want_tokens
        if tag.endswith("perm"):
            assert len(set(want_tokens)) > 8


def test_model_oracle_kv4_stays_close_to_fp16_cache(golden):
    """The quantized cache changes the logits by a bounded amount only (sanity of the
    KV4 branch on the pinned graph; its arithmetic is pinned by the kernel fixtures)."""
    from oracle import qwen3 as oq
    g = golden("qwen3_tiny")
    cfg, weights = golden_model_weights(g, "rtn_perm")
    kscale = torch.full((cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim), 0.6)
    prompt = [int(v) for v in g["rtn_perm.prompt0"]]
    a = oq.OracleQwen3(cfg, weights, kscale=kscale, max_tokens=256, kv_mode="fp16")
    b = oq.OracleQwen3(cfg, weights, kscale=kscale, max_tokens=256, kv_mode="kv4")
    for tok in prompt[:-1]:
        a.forward([tok], "decode")
        b.forward([tok], "decode")
    la, lb = a.forward(prompt[-1:], "decode"), b.forward(prompt[-1:], "decode")
    assert (la - lb).abs().max() / la.pow(2).mean().sqrt() < 0.25
