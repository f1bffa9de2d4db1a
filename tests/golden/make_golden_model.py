"""Regenerate ``qwen3_tiny.npz``: the reference's CPU whole-model path on a tiny Qwen3.

    LINKQ2_REFERENCE=/path/to/LinkQ2 python tests/golden/make_golden_model.py

Everything written is produced by reference code or by HF ``transformers`` driven the
way the reference drives it: a random-init ``Qwen3ForCausalLM`` (the recipe of the
reference's ``tests/conftest.py:25-34``) is quantized by ``quantize_model`` (RTN and
affine), written by ``save_checkpoint``, loaded back dense by
``adapters.model_builder.build_quantized_causal_lm(fake=True)`` on CPU in fp32, and run
for prompt logits and 64 greedy tokens (``generate(do_sample=False)``, as
``tests/runtime/test_execution.py:25-27`` does).  Two heads per checkpoint: the
embedding copied into the LM head (the reference's fixture) and a permuted copy, which
makes greedy decoding walk through many different tokens.  The file keeps the
checkpoint tensors so that the test needs neither the reference nor ``transformers``.
Nothing here calls the oracle or the CUDA kernels.
"""
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

REFERENCE = os.environ.get("LINKQ2_REFERENCE")
if not REFERENCE:
    raise SystemExit("set LINKQ2_REFERENCE to a checkout of the reference (the directory that holds qslab/)")
sys.path.insert(0, REFERENCE)
sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
OUT = Path(__file__).resolve().parent

from transformers import Qwen3Config, Qwen3ForCausalLM  # noqa: E402

from baseline import accelerate_stub  # noqa: E402  (the image has no accelerate package)

accelerate_stub.install()

CFG = dict(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
           num_attention_heads=2, num_key_value_heads=1, head_dim=64, max_position_embeddings=512,
           rms_norm_eps=1e-6, tie_word_embeddings=False)
NEW_TOKENS = 64


def one_case(tag, algorithm, permuted_head, seed, out):
    from adapters.model_builder import build_quantized_causal_lm
    from qslab.compression.checkpoint import save_checkpoint
    from qslab.compression.config import CompressionConfig
    from qslab.compression.pipeline import quantize_model
    from qslab.quantization import QuantizationMethod
    from safetensors import safe_open

    torch.manual_seed(seed)
    hf = Qwen3ForCausalLM(Qwen3Config(rope_theta=1e6, **CFG)).half().eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        embed = (torch.randn(128, 128, generator=g) * 0.5).half()
        hf.model.embed_tokens.weight.copy_(embed)
        for name, p in hf.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_((1 + 0.1 * torch.randn(p.shape, generator=g)).half())
        if permuted_head:
            perm = torch.randperm(128, generator=g)
            head = torch.empty_like(embed)
            head[perm] = embed
            hf.lm_head.weight.copy_(head)
        else:
            hf.lm_head.weight.copy_(embed)
    with tempfile.TemporaryDirectory() as tmp:
        source, quantized = Path(tmp) / "fp16", Path(tmp) / "w4"
        hf.save_pretrained(source)
        calib = [[int(t) for t in torch.randint(0, 127, (16,), generator=g)]]
        artifact = quantize_model(hf, CompressionConfig(algorithm=QuantizationMethod(algorithm), device="cpu"), calib)
        save_checkpoint(artifact, source, quantized)
        dense = build_quantized_causal_lm(quantized, device="cpu", dtype=torch.float32, fake=True)
        prompts = [torch.randint(0, 127, (n,), generator=g).tolist() for n in (23, 9)]
        for i, prompt in enumerate(prompts):
            ids = torch.tensor([prompt])
            with torch.inference_mode():
                logits = dense(input_ids=ids, use_cache=False).logits[0]
                tokens = dense.generate(ids, max_new_tokens=NEW_TOKENS, do_sample=False, eos_token_id=None,
                                        pad_token_id=0)[0, len(prompt):]
            out[f"{tag}.prompt{i}"] = np.array(prompt)
            out[f"{tag}.prompt{i}.logits"] = logits.float().numpy()
            out[f"{tag}.prompt{i}.tokens"] = tokens.numpy()
        with safe_open(str(quantized / "model.safetensors"), framework="pt") as f:
            for name in f.keys():
                t = f.get_tensor(name)
                out[f"{tag}.ckpt.{name}"] = t.numpy()
        out[f"{tag}.config"] = np.frombuffer((quantized / "config.json").read_bytes(), dtype=np.uint8)
        out[f"{tag}.layers"] = np.frombuffer((quantized / "quantized_layers.json").read_bytes(), dtype=np.uint8)


def main():
    out = {}
    one_case("rtn_tied", "rtn_w4a16", False, 7, out)
    one_case("rtn_perm", "rtn_w4a16", True, 8, out)
    one_case("affine_perm", "awq_affine_w4a16", True, 9, out)
    np.savez_compressed(OUT / "qwen3_tiny.npz", **out)
    print("qwen3_tiny.npz", len(out), "arrays", (OUT / "qwen3_tiny.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
