"""Model construction from a complete W4 checkpoint, or from seeded random
weights of the same layout.

Checkpoint layout (``qslab/compression/checkpoint.py:33-63``, read by
``qslab/runtime/quantization.py:15-66``): the original safetensors shards;
``<module>.weight`` int8 logical values, ``.weight.scale`` fp16, optional
``.weight.zero_point`` and ``.weight.input_scale``; ``config.json`` with a
``quantization_config``; ``quantized_layers.json`` listing the swapped modules.
Layout conversion (packing, transposes, tensor-parallel slicing) happens here,
at load time; the files are never rewritten.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn

from linkq2_b200.runtime.backends import make_quant_linear
from linkq2_b200.runtime.model.qwen3 import ModelConfig, Qwen3ForCausalLM
from linkq2_b200.runtime.parallel import COLUMN, ROW, get_tp, shard_dense, shard_quantized

# quant_method -> (symmetric, tensor suffixes beyond '' and '.scale');
# qslab/runtime/quantization_strategies.py:23-62
METHODS = {
    "rtn_w4a16": (True, ()),
    "rtn_clip_w4a16": (True, ()),
    "awq_w4a16": (True, (".input_scale",)),
    "awq_affine_w4a16": (False, (".input_scale", ".zero_point")),
}


class QuantizedWeights:
    def __init__(self, path):
        from safetensors import safe_open
        self.path = Path(path)
        self.model_config = json.loads((self.path / "config.json").read_text())
        self.config = self.model_config["quantization_config"]
        if self.config["bits"] != 4:
            raise ValueError("only W4 checkpoints are supported")
        method = str(self.config["quant_method"])
        if method not in METHODS:
            raise ValueError(f"unknown quantization method: {method}")
        self.symmetric, self.extra = METHODS[method]
        index = self.path / "model.safetensors.index.json"
        if index.exists():
            self.weight_map = json.loads(index.read_text())["weight_map"]
        else:
            with safe_open(str(self.path / "model.safetensors"), framework="pt") as f:
                self.weight_map = {name: "model.safetensors" for name in f.keys()}
        layers = json.loads((self.path / "quantized_layers.json").read_text())
        self.names = [name + ".weight" for name in layers]

    def layer(self, name):
        from safetensors import safe_open
        with safe_open(str(self.path / self.weight_map[name]), framework="pt", device="cpu") as f:
            data = {"values": f.get_tensor(name), "scale": f.get_tensor(name + ".scale"),
                    "zero_point": None, "input_scale": None}
            if ".input_scale" in self.extra:
                data["input_scale"] = f.get_tensor(name + ".input_scale")
            if ".zero_point" in self.extra:
                data["zero_point"] = f.get_tensor(name + ".zero_point")
        return data

    def dequantize(self, data):
        """fp32 dense weight (``quantization_strategies.py:15-20,41-42``): the
        'fake' load path of the reference."""
        scale = data["scale"].float()
        zero = 0 if self.symmetric else data["zero_point"].float().unsqueeze(-1)
        dense = ((data["values"].float().reshape(*scale.shape, -1) - zero)
                 * scale.unsqueeze(-1)).reshape_as(data["values"])
        return dense if data["input_scale"] is None else dense / data["input_scale"].float()


def _split_kind(name: str) -> str | None:
    leaf = name.removesuffix(".weight").rsplit(".", 1)[-1]
    return Qwen3ForCausalLM.TP_SPLIT.get(leaf)


def _set_param(model: nn.Module, name: str, tensor: torch.Tensor) -> None:
    parent_name, _, leaf = name.rpartition(".")
    parent = model.get_submodule(parent_name) if parent_name else model
    setattr(parent, leaf, nn.Parameter(tensor, requires_grad=False))


def _set_module(model: nn.Module, name: str, module: nn.Module) -> None:
    parent_name, _, leaf = name.rpartition(".")
    setattr(model.get_submodule(parent_name) if parent_name else model, leaf, module)


@torch.no_grad()
def load_checkpoint_weights(model, path, *, backend="b200", device="cuda:0", dtype=torch.float16,
                            fake=False):
    """Swap every listed projection for a packed W4 layer and load the rest in
    ``dtype``; returns the number of swapped projections
    (``qslab/runtime/quantization.py:37-66``).  ``fake=True`` loads dequantised
    dense weights instead.  Under tensor parallelism each rank keeps its slice."""
    weights = QuantizedWeights(path)
    tp = get_tp()
    group = weights.config["group_size"]
    for key in weights.names:
        name = key.removesuffix(".weight")
        old = model.get_submodule(name)
        data = weights.layer(key)
        kind = _split_kind(key)
        if kind is not None:
            data = shard_quantized(data, kind, tp, group)
        if tuple(old.weight.shape) != tuple(data["values"].shape):
            raise ValueError(f"weight shape differs: {key}")
        if fake:
            _set_param(model, key, weights.dequantize(data).to(device=device, dtype=dtype))
        else:
            if getattr(old, "bias", None) is not None:
                raise ValueError(f"biased quantized projections are not supported: {name}")
            layer = make_quant_linear(backend, data["values"], data["scale"], group_size=group,
                                      symmetric=weights.symmetric, zero_point=data["zero_point"],
                                      input_scale=data["input_scale"], device=device, dtype=dtype)
            _set_module(model, name, layer)
    suffixes = ("", ".scale") + weights.extra
    auxiliary = {name + suffix for name in weights.names for suffix in suffixes}
    from safetensors import safe_open
    own = dict(model.named_parameters())
    for shard in dict.fromkeys(weights.weight_map.values()):
        with safe_open(str(weights.path / shard), framework="pt", device="cpu") as f:
            for name in f.keys():
                if name in auxiliary or name not in own:
                    continue
                tensor = f.get_tensor(name)
                kind = _split_kind(name)
                if kind is not None:
                    tensor = shard_dense(tensor, kind, tp)
                _set_param(model, name, tensor.to(device=device, dtype=dtype))
    if model.config.tie_word_embeddings:
        model.lm_head.weight = model.model.embed_tokens.weight
    return len(weights.names)


def build_from_checkpoint(path, *, device="cuda:0", max_position=None, fake=False):
    cfg = ModelConfig.from_dict(json.loads((Path(path) / "config.json").read_text()))
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg, max_position, device=device)
    load_checkpoint_weights(model, path, device=device, fake=fake)
    if not fake:
        model.fuse_projections()
        model.shard_head()
    return model.eval()


# ---- seeded random weights in checkpoint layout -----------------------------
def rtn_quantize_(weight: torch.Tensor, group_size: int):
    """Symmetric RTN of ``qslab/compression/algorithms/rtn.py:21-23`` on whatever
    device ``weight`` lives: ``values int8 [N, K]``, ``scale fp16 [N, K/G]``."""
    n, k = weight.shape
    grouped = weight.float().reshape(n, -1, group_size)
    scale = (grouped.abs().amax(-1, keepdim=True) / 7).clamp_min(1e-12)
    values = torch.round(grouped / scale).clamp(-8, 7).to(torch.int8)
    return values.reshape(n, k), scale.squeeze(-1).to(torch.float16)


@torch.no_grad()
def build_random(cfg: ModelConfig, *, seed=0, group_size=128, device="cuda:0", max_position=None,
                 std=0.02, tie_head_to_embedding=True):
    """Random-init model, every decoder projection RTN-W4 quantized exactly as a
    checkpoint of that weight would be.  Each logical ``[N, K]`` weight is drawn
    from its own seeded generator *before* the tensor-parallel slice, so every
    world size computes with the same weights.  ``tie_head_to_embedding`` copies
    the embedding into the LM head, which gives greedy decoding large margins on
    random weights (the trick of the reference's test fixture,
    ``tests/conftest.py:31-34``)."""
    tp = get_tp()
    tp.check_geometry(cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads,
                      cfg.num_key_value_heads, group_size)
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg, max_position, device=device)
    dev = torch.device(device)
    gen = torch.Generator(device=dev)

    def draw(shape, tag):
        gen.manual_seed(seed * 1_000_003 + tag)
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std

    tag = 0
    for name, module in list(model.named_modules()):
        leaf = name.rsplit(".", 1)[-1]
        if leaf not in Qwen3ForCausalLM.TP_SPLIT:
            continue
        tag += 1
        kind = Qwen3ForCausalLM.TP_SPLIT[leaf]
        n_local, k_local = module.weight.shape
        n = n_local * (tp.size if kind == COLUMN else 1)
        k = k_local * (tp.size if kind == ROW else 1)
        w = draw((n, k), tag).to(torch.float16)
        values, scale = rtn_quantize_(w, group_size)
        data = shard_quantized({"values": values, "scale": scale, "zero_point": None,
                                "input_scale": None}, kind, tp, group_size)
        layer = make_quant_linear("b200", data["values"], data["scale"], group_size=group_size,
                                  symmetric=True, device=device, dtype=torch.float16)
        _set_module(model, name, layer)
        del w, values, scale, data
    embed = draw((cfg.vocab_size, cfg.hidden_size), 10_000).to(torch.float16)
    _set_param(model, "model.embed_tokens.weight", embed)
    if cfg.tie_word_embeddings or tie_head_to_embedding:
        model.lm_head.weight = model.model.embed_tokens.weight
    else:
        _set_param(model, "lm_head.weight", draw((cfg.vocab_size, cfg.hidden_size), 10_001).to(torch.float16))
    for name, param in list(model.named_parameters()):
        if param.is_meta:                      # the RMSNorm weights
            _set_param(model, name, torch.ones(param.shape, dtype=torch.float16, device=dev))
    model.fuse_projections()
    model.shard_head()
    return model.eval()


@torch.no_grad()
def save_random_checkpoint(path, cfg: ModelConfig, *, seed: int = 0, group_size: int = 128,
                           weight_std: float = 0.05) -> Path:
    """Write a small seeded RTN-W4 checkpoint in the reference's on-disk layout
    (``qslab/compression/checkpoint.py:33-63``): every tensor is drawn from one CPU
    generator, so the same ``(cfg, seed)`` gives the same files wherever it runs.  The LM
    head is a row permutation of the embedding, which makes greedy decoding on random
    weights walk through many tokens with large margins.  Used by the self-check of
    ``bench.py`` and by tests; real checkpoints come from the reference's offline pipeline."""
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    hid, inter, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    shapes = {"self_attn.q_proj": (hq * d, hid), "self_attn.k_proj": (hkv * d, hid),
              "self_attn.v_proj": (hkv * d, hid), "self_attn.o_proj": (hid, hq * d),
              "mlp.gate_proj": (inter, hid), "mlp.up_proj": (inter, hid), "mlp.down_proj": (hid, inter)}
    tensors, layers = {}, []
    embed = (torch.randn(cfg.vocab_size, hid, generator=g) * 0.5).half()
    tensors["model.embed_tokens.weight"] = embed
    perm = torch.randperm(cfg.vocab_size, generator=g)
    head = torch.empty_like(embed)
    head[perm] = embed
    tensors["lm_head.weight"] = head
    tensors["model.norm.weight"] = torch.ones(hid, dtype=torch.float16)
    for li in range(cfg.num_hidden_layers):
        p = f"model.layers.{li}."
        for nm in ("input_layernorm", "post_attention_layernorm"):
            tensors[p + nm + ".weight"] = (1 + 0.1 * torch.randn(hid, generator=g)).half()
        for nm in ("self_attn.q_norm", "self_attn.k_norm"):
            tensors[p + nm + ".weight"] = (1 + 0.1 * torch.randn(d, generator=g)).half()
        for nm, shape in shapes.items():
            w = (torch.randn(*shape, generator=g) * weight_std).half()
            values, scale = rtn_quantize_(w, group_size)
            tensors[p + nm + ".weight"] = values.contiguous()
            tensors[p + nm + ".weight.scale"] = scale.contiguous()
            layers.append(p + nm)
    save_file(tensors, str(path / "model.safetensors"))
    config = {f: getattr(cfg, f) for f in cfg.__dataclass_fields__}
    config["tie_word_embeddings"] = False
    config["quantization_config"] = {"quant_method": "rtn_w4a16", "bits": 4, "group_size": group_size,
                                     "symmetric": True}
    (path / "config.json").write_text(json.dumps(config))
    (path / "quantized_layers.json").write_text(json.dumps(layers))
    return path
