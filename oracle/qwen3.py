"""CPU oracle for a whole Qwen3 W4 + KV4 forward (test infrastructure, never shipped).

A single-sequence restatement of the reference's layer graph
(``qslab/runtime/model/qwen3.py:43-123``) with dequantised dense weights — what
the reference calls the fake path (``qslab/runtime/quantization.py:45-48``) —
and the KV4 cache arithmetic of :mod:`oracle.kv4`:

* every token's K (after q/k-norm, RoPE and the SmoothAttention division) and V
  are quantized into the cache before attention (``attention.py:102-110``);
* prefill rows attend to the fp16 K/V of their own step and to the dequantised
  cache for earlier steps (``attention.py:112-131``);
* decode and verify rows attend to the dequantised cache only, including their
  own token (``attention.py:132-143``).

Activations are held in fp16 between operators and every operator computes in
fp32, which is where the GPU runtime rounds as well.

Pinned: ``tests/golden/qwen3_tiny.npz`` holds logits and greedy tokens of the
reference's CPU whole-model path (HF ``Qwen3ForCausalLM`` built by
``adapters/model_builder.py:19-30`` with ``fake=True`` weights from a checkpoint
written by the reference's own pipeline); ``kv_mode='fp16'`` runs this restatement
with the cache quantization bypassed, as that model has none, and
``tests/test_oracle_golden.py`` compares the two.  The KV4 arithmetic itself is
pinned by the kernel-level fixtures of :mod:`oracle.kv4`.
"""
from __future__ import annotations

import torch

from . import kv4


def _rms(x, weight, eps):
    x32 = x.float()
    return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).half() * weight


def _rope(x, pos, theta):
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float) / d))
    f = torch.einsum("i,j->ij", pos.float(), inv)
    cos, sin = f.cos().unsqueeze(1), f.sin().unsqueeze(1)
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).half()


class OracleQwen3:
    """``weights``: name -> tensor; projections are dense fp32 ``[N, K]``
    (dequantised), norms/embedding fp16.  ``kscale``/``lam``: ``[L, HKV, D]``."""

    def __init__(self, cfg, weights: dict, kscale: torch.Tensor, lam: torch.Tensor | None = None,
                 v_group: int = 64, max_tokens: int = 4096, kv_mode: str = "kv4"):
        if kv_mode not in ("kv4", "fp16"):
            raise ValueError("kv_mode is 'kv4' or 'fp16'")
        self.cfg, self.w, self.v_group = cfg, weights, v_group
        self.lam = lam
        self.kv_mode = kv_mode
        self.history = [[torch.zeros(0, cfg.num_key_value_heads, cfg.head_dim, dtype=torch.float16)] * 2
                        for _ in range(cfg.num_hidden_layers)]    # fp16 K, V per layer (kv_mode 'fp16')
        self.pools = []
        for layer in range(cfg.num_hidden_layers):
            kc, vc = kv4.empty_pool(max_tokens, cfg.num_key_value_heads, cfg.head_dim, v_group)
            kc[1].copy_(kscale[layer].half())
            self.pools.append((kc, vc))
        self.length = 0                         # tokens in the cache

    def _lin(self, x, name):
        return (x.float() @ self.w[name].float().t()).half()

    def forward(self, token_ids: list[int], mode: str) -> torch.Tensor:
        """Process ``token_ids`` at positions ``length ..``; ``mode`` is 'prefill'
        (fp16 self-chunk attention) or 'decode' (cache-only attention; several
        tokens = a verify step).  Returns fp32 logits ``[T, vocab]``."""
        cfg = self.cfg
        t = len(token_ids)
        pos = torch.arange(self.length, self.length + t)
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        rep = hq // hkv
        h = self.w["model.embed_tokens.weight"][torch.tensor(token_ids)]
        residual = None
        for li in range(cfg.num_hidden_layers):
            p = f"model.layers.{li}."
            if residual is None:
                residual, x = h, _rms(h, self.w[p + "input_layernorm.weight"], cfg.rms_norm_eps)
            else:
                residual = (h.float() + residual.float()).half()
                x = _rms(residual, self.w[p + "input_layernorm.weight"], cfg.rms_norm_eps)
            q = self._lin(x, p + "self_attn.q_proj.weight").view(t, hq, d)
            k = self._lin(x, p + "self_attn.k_proj.weight").view(t, hkv, d)
            v = self._lin(x, p + "self_attn.v_proj.weight").view(t, hkv, d)
            q = _rms(q, self.w[p + "self_attn.q_norm.weight"], cfg.rms_norm_eps)
            k = _rms(k, self.w[p + "self_attn.k_norm.weight"], cfg.rms_norm_eps)
            q, k = _rope(q, pos, cfg.rope_theta), _rope(k, pos, cfg.rope_theta)
            if self.lam is not None:
                lam = self.lam[li].half()
                q = q * lam.repeat_interleave(rep, 0)
                k = k / lam
            kc, vc = self.pools[li]
            end = self.length + t
            if self.kv_mode == "fp16":
                kh, vh = self.history[li]
                self.history[li] = [torch.cat([kh, k]), torch.cat([vh, v])]
                kk, vv = self.history[li][0].float(), self.history[li][1].float()
            else:
                kv4.store_kv_quant(k, v, kc, vc, pos.to(torch.int32), v_group=self.v_group)
            if self.kv_mode == "fp16":
                pass                                  # no cache quantization: every row sees fp16 K/V
            elif mode == "prefill":
                kp, vp = kv4.materialize_kv(kc, vc, torch.arange(self.length), v_group=self.v_group)
                kk = torch.cat([kp, k]).float()
                vv = torch.cat([vp, v]).float()
            else:
                kk, vv = kv4.dequantize_slots(kc, vc, torch.arange(end), v_group=self.v_group)
            heads = torch.arange(hq) // rep
            scores = torch.einsum("thd,shd->hts", q.float(), kk[:, heads]) * d ** -0.5
            mask = torch.arange(end)[None, :] <= pos[:, None]
            scores = scores.masked_fill(~mask[None], float("-inf"))
            o = torch.einsum("hts,shd->thd", torch.softmax(scores, -1), vv[:, heads]).half()
            a = self._lin(o.reshape(t, hq * d), p + "self_attn.o_proj.weight")
            residual = (a.float() + residual.float()).half()
            x = _rms(residual, self.w[p + "post_attention_layernorm.weight"], cfg.rms_norm_eps)
            gate = self._lin(x, p + "mlp.gate_proj.weight")
            up = self._lin(x, p + "mlp.up_proj.weight")
            act = (torch.nn.functional.silu(gate.float()).half() * up)
            h = self._lin(act, p + "mlp.down_proj.weight")
        self.length += t
        final = _rms((h.float() + residual.float()).half(), self.w["model.norm.weight"], cfg.rms_norm_eps)
        self.last_logits = final.float() @ self.w["lm_head.weight"].float().t()
        return self.last_logits

    def greedy(self, prompt: list[int], new_tokens: int, chunk: int | None = None) -> list[int]:
        chunk = chunk or len(prompt)
        logits = None
        for i in range(0, len(prompt), chunk):
            logits = self.forward(prompt[i:i + chunk], "prefill")
        out = [int(logits[-1].argmax())]
        for _ in range(new_tokens - 1):
            out.append(int(self.forward([out[-1]], "decode")[-1].argmax()))
        return out
