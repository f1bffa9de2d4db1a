"""Run the unmodified LinkQ2 reference (installed under ``baseline/_ref`` by
``install_reference.sh``) on this GPU, next to this library, and record what comes out.

    python baseline/reference_gpu.py tests     # the reference's own GPU tests: stock, then with the
                                               # operators rebound to this library (the drop-in proof)
    python baseline/reference_gpu.py tokens    # greedy tokens, reference runtime (w4 + kv4, graphs) vs this runtime
    python baseline/reference_gpu.py store     # KV4 store: reference Triton kernel on the GPU vs the IEEE oracle
    python baseline/reference_gpu.py kernels   # device time of the reference's Triton kernels and of this library's
    python baseline/reference_gpu.py all

Every section prints one JSON line and appends it to ``reference_gpu.jsonl`` in the output directory
(``--out``, default ``baseline/out``, or the environment variable ``LINKQ2_REFERENCE_OUT``); a section
that cannot run records the error text instead (that text is then the result).  Nothing here is
imported by the package, the tests or ``bench.py``.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
import traceback
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
for p in (str(HERE / "_ref"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)
OUT = Path(os.environ.get("LINKQ2_REFERENCE_OUT", HERE / "out"))


def emit(section: str, payload: dict) -> None:
    OUT.mkdir(parents=True, exist_ok=True)
    line = json.dumps({"section": section, **payload})
    print(line, flush=True)
    with open(OUT / "reference_gpu.jsonl", "a") as f:
        f.write(line + "\n")


def prepare(hf_compat: bool = True):
    from baseline import accelerate_stub, dropin_plugin
    accelerate_stub.install()
    if hf_compat:
        dropin_plugin.hf_compat()
    return dropin_plugin


# --------------------------------------------------------------------------- tests
REF_TESTS = ["kernels/test_kv4_paged.py", "kernels/test_kv4_verify.py", "kernels/test_kv4_materialize.py",
             "kernels/test_w4a16.py", "runtime/test_attention.py", "speculation/test_ngram_execution.py"]


def run_pytest(env_extra: dict, tag: str) -> dict:
    env = dict(os.environ, **env_extra)
    paths = [str(HERE / "_ref" / "reference_tests" / t) for t in REF_TESTS]
    cmd = [sys.executable, "-m", "pytest", "-p", "baseline.dropin_plugin", "-m", "gpu", "-rA", "-q",
           "--no-header", "-p", "no:cacheprovider", "--timeout", "600", *paths]
    res = subprocess.run(cmd, cwd=str(ROOT), env=env, capture_output=True, text=True)
    (OUT / f"reference_tests_{tag}.log").write_text(res.stdout[-200000:] + "\n--- stderr\n" + res.stderr[-20000:])
    outcome = {}
    for row in res.stdout.splitlines():
        for word in ("PASSED", "FAILED", "ERROR", "SKIPPED"):
            if row.startswith(word + " "):
                name = row[len(word) + 1:].split(" - ")[0].strip()
                outcome[name.split("reference_tests/")[-1]] = word
    tail = [r for r in res.stdout.strip().splitlines()[-3:]]
    return {"exit": res.returncode, "summary": tail[-1] if tail else "", "outcomes": outcome}


def section_tests(_args):
    OUT.mkdir(parents=True, exist_ok=True)
    stock = run_pytest({}, "stock")
    emit("tests.stock", {"what": "reference tests, reference kernels, image as is", **stock})
    compat = run_pytest({"LINKQ2_HF_COMPAT": "1"}, "stock_hf_compat")
    emit("tests.stock_hf_compat", {"what": "same with the transformers-5 config view", **compat})
    dropin = run_pytest({"LINKQ2_HF_COMPAT": "1", "LINKQ2_DROPIN": "1", "LINKQ2_DROPIN_GEMLITE": "1"}, "dropin")
    emit("tests.dropin", {"what": "reference tests with qslab.kernels.kv4 and the quant backend rebound to linkq2_b200",
                          **dropin})


# --------------------------------------------------------------------------- tokens
GEOMETRY = {
    "tiny": dict(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                 num_attention_heads=2, num_key_value_heads=1, head_dim=64, max_position_embeddings=4096,
                 tie_word_embeddings=True),
    "1p7b": dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                 num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                 tie_word_embeddings=True),
    "1p7b_permuted_head": dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                               num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                               max_position_embeddings=40960, tie_word_embeddings=False),
}


def build_checkpoint(geometry: str, layers: int | None, work: Path, seed: int = 7):
    """Random-init HF Qwen3 -> the reference's RTN-W4 g128 checkpoint + a unit-lambda calibration,
    with the reference's own offline pipeline."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from qslab.compression.checkpoint import save_checkpoint
    from qslab.compression.config import CompressionConfig
    from qslab.compression.pipeline import quantize_model
    kw = dict(GEOMETRY[geometry])
    if layers:
        kw["num_hidden_layers"] = layers
    cfg = Qwen3Config(rope_theta=1e6, **kw)
    torch.manual_seed(seed)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    with torch.device(dev):
        hf = Qwen3ForCausalLM(cfg).half().eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        if kw["tie_word_embeddings"]:
            hf.lm_head.weight = hf.model.embed_tokens.weight
        else:
            # Random-init layers give nearly flat logits whose arg-max is decided by rounding noise in any
            # implementation.  A larger embedding and a head that is a row permutation of it make greedy
            # decoding walk through the vocabulary with margins that numerics cannot flip, while attention
            # and the MLPs still shape the logits (compared numerically as well).
            embed = (torch.randn(kw["vocab_size"], kw["hidden_size"], generator=g) * 0.5).half()
            perm = torch.randperm(kw["vocab_size"], generator=g)
            head = torch.empty_like(embed)
            head[perm] = embed
            hf.model.embed_tokens.weight.copy_(embed)
            hf.lm_head.weight.copy_(head)
            for name, param in hf.named_parameters():       # small residual branches: the embedding stays dominant
                if name.endswith(("o_proj.weight", "down_proj.weight")):
                    param.mul_(0.05)
    source, quantized = work / "fp16", work / "w4"
    hf.save_pretrained(source)
    artifact = quantize_model(hf, CompressionConfig(group_size=128, device=dev))
    save_checkpoint(artifact, source, quantized)
    del hf, artifact
    torch.cuda.empty_cache()
    calibration = work / "kv4.pt"
    shape = (kw["num_hidden_layers"], kw["num_key_value_heads"], kw["head_dim"])
    torch.save({"lambda": torch.ones(shape), "kscale": torch.full(shape, 0.5)}, calibration)
    return quantized, calibration, kw


def reference_generate(quantized, calibration, prompt, new_tokens, vocab, max_len):
    """The reference's LLMEngine on its stock path: quant_backend 'gemlite', kv4, CUDA graphs."""
    import torch
    from types import SimpleNamespace
    import qslab.runtime.engine.llm_engine as eng
    from qslab.runtime.sampling_params import SamplingParams
    eng.AutoTokenizer.from_pretrained = staticmethod(lambda *a, **k: SimpleNamespace(
        eos_token_id=vocab - 1, all_special_ids=[vocab - 1], get_vocab=lambda: {}))
    engine = eng.LLMEngine(str(quantized), kv_cache_dtype="kv4", smooth_kv=str(calibration), enforce_eager=False,
                           max_num_seqs=1, max_model_len=max_len, max_num_batched_tokens=max(len(prompt), 64),
                           num_kvcache_blocks=(max_len + 255) // 256 + 1, kvcache_block_size=256)
    logits = []
    hook = engine.model_runner.model.lm_head.register_forward_hook(lambda m, i, o: logits.append(o.detach().float().cpu()))
    try:
        seq = engine.add_request(list(prompt), SamplingParams(max_tokens=new_tokens, temperature=0, ignore_eos=True))
        engine.step()                                   # prefill + first token
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        steps = 0
        while not engine.is_finished():
            engine.step()
            steps += 1
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        tokens = list(seq.completion_token_ids)
    finally:
        hook.remove()
        engine.exit()
    return tokens, dt / max(steps, 1) * 1e3, logits


def ours_generate(quantized, kscale, kw, prompt, new_tokens, max_len):
    import torch
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig
    from linkq2_b200.runtime.quantization import build_from_checkpoint
    from linkq2_b200.runtime.state import BlockPool, Sequence
    model = build_from_checkpoint(quantized, device="cuda:0", max_position=max_len + 64)
    blocks = (max_len + 255) // 256 + 1
    rc = RunnerConfig(kvcache_block_size=256, num_kvcache_blocks=blocks, max_num_seqs=1, max_model_len=max_len,
                      enforce_eager=False)
    shape = (kw["num_hidden_layers"], kw["num_key_value_heads"], kw["head_dim"])
    runner = ModelRunner(model, rc, smooth_kv={"lambda": torch.ones(shape), "kscale": torch.full(shape, kscale)},
                         device="cuda:0")
    runner.keep_logits = True
    seq = Sequence(list(prompt), 256)
    BlockPool(blocks).ensure(seq, len(prompt) + new_tokens + 8)
    first = runner.run([seq], True)
    first_logits = runner.last_logits.float().cpu()
    seq.append(first[0])
    tokens = [first[0]]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(new_tokens - 1):
        tok = runner.run([seq], False)
        seq.append(tok[0])
        tokens.append(tok[0])
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    last_logits = runner.last_logits.float().cpu()
    runner.shutdown()
    return tokens, dt / max(new_tokens - 1, 1) * 1e3, first_logits, last_logits


def ours_follow(quantized, kscale, kw, prompt, forced, max_len):
    """This library's runtime fed with the reference's tokens (teacher forcing): at every step the
    margin, in units of the logits' RMS, by which this runtime's top logit exceeds its logit of the
    token the reference chose (0 where both choose the same token)."""
    import torch
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig
    from linkq2_b200.runtime.quantization import build_from_checkpoint
    from linkq2_b200.runtime.state import BlockPool, Sequence
    model = build_from_checkpoint(quantized, device="cuda:0", max_position=max_len + 64)
    blocks = (max_len + 255) // 256 + 1
    rc = RunnerConfig(kvcache_block_size=256, num_kvcache_blocks=blocks, max_num_seqs=1, max_model_len=max_len,
                      enforce_eager=False)
    shape = (kw["num_hidden_layers"], kw["num_key_value_heads"], kw["head_dim"])
    runner = ModelRunner(model, rc, smooth_kv={"lambda": torch.ones(shape), "kscale": torch.full(shape, kscale)},
                         device="cuda:0")
    runner.keep_logits = True
    seq = Sequence(list(prompt), 256)
    BlockPool(blocks).ensure(seq, len(prompt) + len(forced) + 8)
    margins = []
    for i, token in enumerate(forced):
        runner.run([seq], i == 0)
        logits = runner.last_logits.float()[-1]
        margins.append(float((logits.max() - logits[token]) / logits.pow(2).mean().sqrt()))
        seq.append(token)
    runner.shutdown()
    return margins


def section_tokens(args):
    import tempfile
    import torch
    prepare()
    cases = (("tiny", None, 40, 64), ("1p7b", args.layers, 512, 256), ("1p7b_permuted_head", args.layers, 512, 256))
    for geometry, layers, prompt_len, new_tokens in cases:
        if args.only and geometry != args.only:
            continue
        rec = {"geometry": geometry, "prompt_tokens": prompt_len, "new_tokens": new_tokens}
        try:
            with tempfile.TemporaryDirectory() as tmp:
                t0 = time.time()
                quantized, calibration, kw = build_checkpoint(geometry, layers, Path(tmp))
                rec["layers"] = kw["num_hidden_layers"]
                rec["build_s"] = round(time.time() - t0, 1)
                g = torch.Generator().manual_seed(11)
                prompt = torch.randint(0, kw["vocab_size"] - 1, (prompt_len,), generator=g).tolist()
                max_len = (prompt_len + new_tokens + 8 + 255) // 256 * 256
                ours, ours_ms, ours_first, ours_last = ours_generate(quantized, 0.5, kw, prompt, new_tokens, max_len)
                rec.update(ours_tokens=ours[:64], ours_tpot_ms=round(ours_ms, 3), distinct_tokens=len(set(ours)))
                try:
                    ref, ref_ms, ref_logits = reference_generate(quantized, calibration, prompt, new_tokens,
                                                                 kw["vocab_size"], max_len)
                    n = min(len(ref), len(ours))
                    same = next((i for i in range(n) if ref[i] != ours[i]), n)
                    rec.update(reference_tokens=ref[:64], reference_tpot_ms=round(ref_ms, 3),
                               identical_prefix=same, first_64_identical=bool(same >= min(64, n)),
                               all_identical=bool(ref[:n] == ours[:n]))
                    if same < n:
                        # random-init logits are nearly flat, so one near-tie sends two correct runs apart;
                        # follow the reference's tokens and measure every disagreement
                        margins = ours_follow(quantized, 0.5, kw, prompt, ref[:64], max_len)
                        off = [m for m in margins if m > 0]
                        rec.update(forced_steps=len(margins), forced_disagreements=len(off),
                                   forced_max_margin_over_rms=round(max(off), 5) if off else 0.0)
                    if ref_logits:
                        a, b = ref_logits[0][-1], ours_first[-1]
                        rec["first_logits_err_over_rms"] = round(float((a - b).abs().max() / b.pow(2).mean().sqrt()), 5)
                        a, b = ref_logits[-1][-1], ours_last[-1]
                        rec["last_logits_err_over_rms"] = round(float((a - b).abs().max() / b.pow(2).mean().sqrt()), 5)
                except Exception as e:                          # the error text is the result
                    rec["reference_error"] = f"{type(e).__name__}: {e}"[:2000]
                    rec["reference_traceback_tail"] = traceback.format_exc()[-1500:]
        except Exception as e:
            rec["error"] = f"{type(e).__name__}: {e}"[:2000]
            rec["traceback_tail"] = traceback.format_exc()[-1500:]
        emit("tokens", rec)


# --------------------------------------------------------------------------- store
def section_store(_args):
    import torch
    prepare()
    from oracle import kv4 as ok
    rec = {}
    try:
        from qslab.kernels.kv4 import store_kv_quant as ref_store
        from linkq2_b200.kernels.kv4 import store_kv_quant as our_store
        tokens, hkv, d = 8192, 8, 128
        k, v = ok.seeded_kv(tokens, hkv, d, 2026)
        ks = ok.static_k_scale(k)
        slots = torch.randperm(tokens, generator=torch.Generator().manual_seed(3)).int()
        pools = {}
        for name in ("oracle", "reference", "ours"):
            kc, vc = ok.empty_pool(tokens, hkv, d, 64)
            kc[1].copy_(ks)
            if name != "oracle":
                kc = (kc[0].cuda(), kc[1].cuda())
                vc = (vc[0].cuda(), vc[1].cuda())
            pools[name] = (kc, vc)
        ok.store_kv_quant(k, v, *pools["oracle"], slots, v_group=64)
        ref_store(k.cuda(), v.cuda(), *pools["reference"], slots.cuda(), v_group=64)
        our_store(k.cuda(), v.cuda(), *pools["ours"], slots.cuda(), v_group=64)
        torch.cuda.synchronize()

        def nibbles(words):
            w = words.cpu().view(torch.int32).long() & 0xFFFFFFFF
            return torch.stack([(w >> (4 * j)) & 15 for j in range(8)], -1).flatten()

        total = tokens * hkv * d
        for name in ("reference", "ours"):
            kq = nibbles(pools[name][0][0]); vq = nibbles(pools[name][1][0])
            okq = nibbles(pools["oracle"][0][0]); ovq = nibbles(pools["oracle"][1][0])
            rec[f"{name}_k_code_mismatches"] = int((kq != okq).sum())
            rec[f"{name}_v_code_mismatches"] = int((vq != ovq).sum())
            rec[f"{name}_v_scale_mismatches"] = int((pools[name][1][1].cpu().view(torch.int16)
                                                     != pools["oracle"][1][1].view(torch.int16)).sum())
            rec[f"{name}_max_code_distance"] = int(max((kq - okq).abs().max(), (vq - ovq).abs().max()))
        rec["codes_per_tensor"] = total
        rec["what"] = ("K/V ~ N(0,1) fp16, 4 outlier channels per head x10, static K scale amax/7; codes compared with the "
                       "IEEE-division CPU oracle")
    except Exception as e:
        rec["error"] = f"{type(e).__name__}: {e}"[:2000]
        rec["traceback_tail"] = traceback.format_exc()[-1500:]
    emit("store", rec)


# --------------------------------------------------------------------------- kernels
def time_graph(calls, reps=20):
    """Median device time per call (us): the calls, over distinct inputs whose total exceeds L2,
    captured into one CUDA graph and replayed; CUDA events on the replaying stream."""
    import torch
    side = torch.cuda.Stream()
    with torch.cuda.stream(side), torch.inference_mode():
        for c in calls:
            c()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for c in calls:
                c()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(side)
            graph.replay()
            b.record(side)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
    return sorted(times)[len(times) // 2] * 1e3 / len(calls)


def section_kernels(args):
    import torch
    prepare()
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
        else {"hbm_gbs": 6650.0}
    g = torch.Generator().manual_seed(2026)
    # ---- W4A16: config 1 (4096^2, affine g128) and the gate_up shape, M = 1 / 32 / 2048
    for (k, n, affine, ms) in ((4096, 4096, True, (1,)), (4096, 24576, False, (1, 32, 2048)),
                               (4096, 4096, False, (32,))):
        try:
            from qslab.runtime.backends.gemlite import GemLiteLinear
            from linkq2_b200.runtime.backends.b200 import B200Linear
            copies = max(4, int(200e6 // (k * n // 2)) + 1)       # weight set > L2
            codes = torch.randint(0 if affine else -8, 16 if affine else 8, (n, k), generator=g, dtype=torch.int8)
            scale = (torch.rand(n, k // 128, generator=g) * 0.01 + 0.001).half()
            zero = torch.randint(0, 16, scale.shape, generator=g).half() if affine else None
            kw = dict(group_size=128, symmetric=not affine, zero_point=zero, device="cuda", dtype=torch.float16)
            layers = {}
            for name, cls in (("reference", GemLiteLinear), ("ours", B200Linear)):
                try:
                    layers[name] = [cls.from_quantized(codes, scale, **kw) for _ in range(copies)]
                except Exception as e:
                    layers[name] = f"{type(e).__name__}: {e}"[:500]
            for m in ms:
                x = torch.randn(m, k, device="cuda", dtype=torch.float16)
                nbytes = k * n // 2 + (4 if affine else 2) * (k // 128) * n + 2 * m * (k + n)
                rec = {"op": "w4a16", "k": k, "n": n, "m": m, "affine": affine, "copies": copies,
                       "algorithmic_bytes": nbytes, "flops": 2 * m * k * n}
                for name, ls in layers.items():
                    if isinstance(ls, str):
                        rec[name + "_error"] = ls
                        continue
                    try:
                        us = time_graph([lambda l=l: l(x) for l in ls])
                        rec[name + "_us"] = round(us, 2)
                        rec[name + "_gbs"] = round(nbytes / us / 1e3, 1)
                        rec[name + "_frac_hbm"] = round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4)
                        rec[name + "_tflops"] = round(2 * m * k * n / us / 1e6, 1)
                    except Exception as e:
                        rec[name + "_error"] = f"{type(e).__name__}: {e}"[:500]
                emit("kernels", rec)
            del layers
            torch.cuda.empty_cache()
        except Exception as e:
            emit("kernels", {"op": "w4a16", "k": k, "n": n, "error": f"{type(e).__name__}: {e}"[:1000]})
    # ---- KV4 decode and verify
    hq, hkv, d, page = 32, 8, 128, 256
    for (bs, ctx, m) in ((64, 4096, 1), (32, 2304, 1), (32, 2304, 16), (8, 16384, 1)):
        try:
            from qslab.kernels.kv4 import paged_attention_decode as ref_attn
            from linkq2_b200.kernels.kv4 import paged_attention_decode as our_attn
            nb = bs * (ctx // page)
            slots = nb * page
            kq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
            vq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
            ks = (torch.rand(hkv, d, device="cuda") * 0.1 + 0.05).half()
            vs = (torch.rand(slots, hkv, 2, device="cuda") * 0.1 + 0.05).half()
            table = torch.randperm(nb, generator=g).int().view(bs, -1).cuda()
            q = (torch.randn(bs * m, hq, d, device="cuda") * 0.5).half()
            lens = torch.full((bs,), ctx - (m - 1), dtype=torch.int32, device="cuda")
            nbytes = bs * ctx * hkv * (d + 2 * (d // 64)) + 4 * bs * m * hq * d
            rec = {"op": "kv4_attention", "batch": bs, "context": ctx, "verify_m": m, "algorithmic_bytes": nbytes,
                   "cache_mb": round(nbytes / 1e6, 1)}
            outs = {}
            for name, fn in (("reference", ref_attn), ("ours", our_attn)):
                try:
                    call = lambda fn=fn: fn(q, (kq.view(torch.uint32) if fn is ref_attn else kq, ks),
                                            (vq.view(torch.uint32) if fn is ref_attn else vq, vs), table, lens,
                                            block_n=page, num_kv_heads=hkv, v_group=64, verify_m=m)
                    outs[name] = call().float()
                    us = time_graph([call] * 3, reps=10)
                    rec[name + "_us"] = round(us, 2)
                    rec[name + "_gbs"] = round(nbytes / us / 1e3, 1)
                    rec[name + "_frac_hbm"] = round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4)
                except Exception as e:
                    rec[name + "_error"] = f"{type(e).__name__}: {e}"[:500]
            if len(outs) == 2:
                rec["max_abs_diff"] = round(float((outs["reference"] - outs["ours"]).abs().max()), 6)
            emit("kernels", rec)
            del kq, vq, vs
            torch.cuda.empty_cache()
        except Exception as e:
            emit("kernels", {"op": "kv4_attention", "batch": bs, "context": ctx, "error": f"{type(e).__name__}: {e}"[:1000]})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("section", choices=["tests", "tokens", "store", "kernels", "all"])
    ap.add_argument("--layers", type=int, default=None, help="decoder layers of the 1.7B-geometry checkpoint (default 28)")
    ap.add_argument("--only", default=None, help="tokens: run this geometry only")
    ap.add_argument("--out", default=None, help="directory for reference_gpu.jsonl and the test logs")
    args = ap.parse_args()
    if args.out:
        global OUT
        OUT = Path(args.out)
    if not (HERE / "_ref" / "qslab").exists():
        emit(args.section, {"error": "baseline/_ref is missing: run baseline/install_reference.sh first"})
        return
    for name in (["tests", "tokens", "store", "kernels"] if args.section == "all" else [args.section]):
        try:
            {"tests": section_tests, "tokens": section_tokens, "store": section_store,
             "kernels": section_kernels}[name](args)
        except Exception as e:
            emit(name, {"error": f"{type(e).__name__}: {e}"[:2000], "traceback_tail": traceback.format_exc()[-1500:]})


if __name__ == "__main__":
    main()
