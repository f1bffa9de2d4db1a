"""Regenerate ``tp_parity.npz``: greedy tokens and final logits of the CPU oracle model on the
seeded self-check checkpoint that ``bench.py`` decodes on every rank count.

    python tests/golden/make_tp_parity.py

The checkpoint comes from ``linkq2_b200.runtime.quantization.save_random_checkpoint`` (one
CPU generator, so the files are the same on every machine); the oracle (pinned to the
reference's CPU model path by ``qwen3_tiny.npz``) runs on its dequantised weights.  Geometry:
8 query and 8 KV heads of 128 channels, hidden 256, intermediate 1024, 2 layers - the
smallest shape that shards over 8 ranks in groups of 128.
"""
import json
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent

SELF_CHECK = dict(vocab_size=256, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                  num_attention_heads=8, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                  max_position_embeddings=1024, tie_word_embeddings=False)
SEED, KSCALE, NEW_TOKENS, PROMPT_LENS = 21, 0.5, 32, (37, 12, 64, 5)


def main():
    from safetensors import safe_open
    from linkq2_b200.runtime.model.qwen3 import ModelConfig
    from linkq2_b200.runtime.quantization import save_random_checkpoint
    from oracle import qwen3 as oq, w4a16 as ow
    cfg = ModelConfig.from_dict(SELF_CHECK)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        path = save_random_checkpoint(Path(tmp) / "w4", cfg, seed=SEED)
        layers = json.loads((path / "quantized_layers.json").read_text())
        weights = {}
        with safe_open(str(path / "model.safetensors"), framework="pt") as f:
            names = set(f.keys())
            for name in layers:
                key = name + ".weight"
                weights[key] = ow.dequantize_fp32(f.get_tensor(key), f.get_tensor(key + ".scale"), symmetric=True)
            for name in names:
                if name.endswith(".weight") and name not in weights:
                    weights[name] = f.get_tensor(name)
    g = torch.Generator().manual_seed(SEED + 1)
    kscale = torch.full((cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim), KSCALE)
    for i, n in enumerate(PROMPT_LENS):
        prompt = torch.randint(0, cfg.vocab_size - 1, (n,), generator=g).tolist()
        oracle = oq.OracleQwen3(cfg, weights, kscale=kscale, max_tokens=256)
        tokens = oracle.greedy(prompt, NEW_TOKENS)
        out[f"prompt{i}"] = np.array(prompt)
        out[f"tokens{i}"] = np.array(tokens)
        out[f"logits{i}"] = oracle.last_logits[-1].numpy()
        print(i, len(set(tokens)), "distinct tokens")
    out["config"] = np.frombuffer(json.dumps(SELF_CHECK).encode(), dtype=np.uint8)
    out["meta"] = np.array([SEED, NEW_TOKENS, len(PROMPT_LENS)])
    out["kscale"] = np.array([KSCALE])
    np.savez_compressed(OUT / "tp_parity.npz", **out)
    print("tp_parity.npz", (OUT / "tp_parity.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
