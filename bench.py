"""Qwen3-8B W4 + KV4 batched decode throughput on N B200s (tensor parallel), with
the W4A16 kernel's HBM roofline and the CPU restatement timed beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 is launched with ``python -m torch.distributed.run --nproc-per-node N``;
one rank per GPU.  Workload: Qwen3-8B geometry, seeded random weights RTN-W4
group 128, KV4 cache; batch 32, 2048-token prompts (seeded uniform ids) prefilled
in 64-token chunks, then timed single-token decode steps through CUDA graphs, and
one 16-position verify pass.  A step is one decode forward of the whole batch
(one new token per sequence).  Inputs are synthetic; decode reads ~3.3 GB of
weights and ~2.8 GB of KV per step, far more than the 126 MB L2.

``value``  tokens/s with the step's metadata staged on the device and tokens fed
           back device-to-device (no host copies in the timed region).
``e2e``    tokens/s through ``ModelRunner.run``: host lists -> pinned H2D ->
           graph replay -> LM head -> argmax -> D2H token list, every step.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, PROMPT, CHUNK, VERIFY_M = 32, 2048, 64, 16
METRIC, UNIT = "qwen3_8b_w4_kv4_decode_tokens_per_s", "tokens/s"


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return json.loads(f.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ----------------------------------------------------------------------------
# CPU arm: the oracle (a port of the reference's CPU torch path) on host cores
# ----------------------------------------------------------------------------
def cpu_step_sample(cfg, seqs_sampled: int, context: int, threads: int, seed: int = 0):
    """One decoder layer of the reference's CPU path at the bench's decode shape:
    the seven projections as pre-dequantised dense fp32 matmuls at M = 32 (what
    the reference's fake-weight model runs per step) plus KV4 store + paged
    decode through the torch restatement for ``seqs_sampled`` of the 32
    sequences.  Returns a closure timing one such layer."""
    import torch
    from oracle import kv4 as ok, w4a16 as ow
    torch.set_num_threads(threads)
    hid, inter = cfg.hidden_size, cfg.intermediate_size
    hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    shapes = [(hq * d, hid), (hkv * d, hid), (hkv * d, hid), (hid, hq * d), (inter, hid), (inter, hid), (hid, inter)]
    dense = []
    for i, (n, k) in enumerate(shapes):
        values, scale = ow.rtn_quantize(ow.seeded_weight(n, k, seed + i), 128)
        dense.append(ow.dequantize_fp32(values, scale, symmetric=True))
    xs = [ow.seeded_activation(BATCH, k, seed + 50 + i).float() for i, (_, k) in enumerate(shapes)]
    page = 256
    blocks = (context + page) // page
    slots = seqs_sampled * blocks * page
    k, v = ok.seeded_kv(slots, hkv, d, seed)
    kc, vc = ok.empty_pool(slots, hkv, d, 64)
    kc[1].copy_(ok.static_k_scale(k))
    ok.store_kv_quant(k, v, kc, vc, torch.arange(slots), v_group=64)
    table = torch.arange(seqs_sampled * blocks, dtype=torch.int32).view(seqs_sampled, blocks)
    lens = torch.full((seqs_sampled,), context, dtype=torch.int32)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(seqs_sampled, hq, d, generator=g).half()
    k_new, v_new = k[:seqs_sampled].clone(), v[:seqs_sampled].clone()
    new_slots = (table[:, (context - 1) // page].long() * page + (context - 1) % page).int()

    def layer():
        t0 = time.perf_counter()
        for w, x in zip(dense, xs):
            (x @ w.t()).half()
        t1 = time.perf_counter()
        ok.store_kv_quant(k_new, v_new, kc, vc, new_slots, v_group=64)
        ok.paged_attention_decode(q, kc, vc, table, lens, block_n=page, num_kv_heads=hkv, v_group=64)
        t2 = time.perf_counter()
        return t1 - t0, (t2 - t1) * (BATCH / seqs_sampled)
    return layer


def cpu_tokens_per_s(cfg, context, steps, warmup, threads):
    import torch
    sampled = 2
    layer = cpu_step_sample(cfg, sampled, context, threads)
    g = torch.Generator().manual_seed(1)
    head = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * 0.02)
    xh = torch.randn(BATCH, cfg.hidden_size, generator=g)
    for _ in range(max(1, warmup)):
        layer()
    times = []
    for _ in range(steps):
        lin, att = layer()
        t0 = time.perf_counter()
        (xh @ head.t()).argmax(-1)
        th = time.perf_counter() - t0
        times.append(cfg.num_hidden_layers * (lin + att) + th)
    step = sum(times) / len(times)
    sample = (f"per step: 1 of {cfg.num_hidden_layers} decoder layers (7 dense fp32 projections at M={BATCH}, "
              f"KV4 store+decode for {sampled} of {BATCH} sequences at context {context}, scaled x{BATCH // sampled}) "
              f"+ fp32 LM head; step time = {cfg.num_hidden_layers} x layer + head")
    return BATCH / step, step * 1e3, sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from linkq2_b200.runtime.model.qwen3 import ModelConfig
    import torch
    cfg = ModelConfig.qwen3_8b()
    threads = os.cpu_count() or 1
    steps = max(1, min(args.steps, 16))
    value, ms, sample = cpu_tokens_per_s(cfg, PROMPT + 256, steps, min(args.warmup, 2), threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": min(args.warmup, 2), "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + f"; {steps} timed samples"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def workload_config(n_gpus):
    return {"workload": "configs[4]: Qwen3-8B geometry (36 layers, hidden 4096, inter 12288, 32 q / 8 kv heads, "
                        "head_dim 128, vocab 151936), random init RTN-W4 g128 + KV4 (page 256, v_group 64)",
            "batch": BATCH, "prompt_tokens": PROMPT, "prefill": f"chunked, {CHUNK} tokens per sequence per step (untimed)",
            "step": "one decode forward: 32 sequences x 1 new token, CUDA graph + fp16 LM head + argmax",
            "parallelism": f"tp{n_gpus}", "l2": "per-step working set (3.3 GB weights + KV) exceeds the 126 MB L2"}


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            pass

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for row in out.strip().splitlines():
            f = [c.strip() for c in row.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_b200(args):
    import torch
    import torch.distributed as dist
    from linkq2_b200 import _lib
    from linkq2_b200.runtime import parallel
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig, amax_calibration
    from linkq2_b200.runtime.model.context import reset_context, set_context
    from linkq2_b200.runtime.model.qwen3 import ModelConfig
    from linkq2_b200.runtime.quantization import build_random
    from linkq2_b200.runtime.state import BlockPool, Sequence

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device; the operators have no CPU path")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    tp = parallel.init_from_env()
    rank, world = tp.rank, tp.size
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE is {world}")

    cfg = ModelConfig.qwen3_8b()
    steps, warmup = args.steps, max(args.warmup, 3)
    max_len = PROMPT + warmup + steps + VERIFY_M + 8
    max_len = (max_len + 255) // 256 * 256
    page = 256
    blocks_per_seq = max_len // page
    rc = RunnerConfig(kvcache_block_size=page, num_kvcache_blocks=BATCH * blocks_per_seq + 4, v_group=64,
                      max_num_seqs=BATCH, max_model_len=max_len, enforce_eager=False,
                      spec_num_drafts=VERIFY_M - 1)
    t_build = time.time()
    model = build_random(cfg, seed=0, group_size=128, device=device, max_position=max_len + 64)
    runner = ModelRunner(model, rc, device=device,
                         smooth_kv=amax_calibration(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim, 0.5))
    torch.cuda.synchronize()
    t_build = time.time() - t_build

    # ---- prompts and chunked prefill (untimed)
    g = torch.Generator().manual_seed(1234)
    pool = BlockPool(rc.num_kvcache_blocks, shuffle_seed=7)
    seqs = []
    for _ in range(BATCH):
        s = Sequence(torch.randint(0, cfg.vocab_size, (PROMPT,), generator=g).tolist(), page)
        pool.ensure(s, max_len)
        seqs.append(s)
    t_prefill = time.time()
    first = None
    for start in range(0, PROMPT, CHUNK):
        first = runner.run(seqs, True, counts=[CHUNK] * BATCH)
    for s, tok in zip(seqs, first):
        s.append(tok)
    torch.cuda.synchronize()
    t_prefill = time.time() - t_prefill

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def e2e_steps(n):
        for _ in range(n):
            toks = runner.run(seqs, False)
            for s, tok in zip(seqs, toks):
                s.append(tok)

    e2e_steps(warmup)

    # ---- value: K steps, metadata resident on the device
    graphs = runner.cuda_graphs
    base_len = len(seqs[0])
    bt = runner.prepare_block_tables(seqs)
    pos_all = torch.tensor([[base_len - 1 + i] * BATCH for i in range(steps)], dtype=torch.int64, device=device)
    slot_all = torch.tensor([[s.slot(base_len - 1 + i) for s in seqs] for i in range(steps)],
                            dtype=torch.int32, device=device)
    len_all = torch.tensor([[base_len + i] * BATCH for i in range(steps)], dtype=torch.int32, device=device)
    ids = torch.tensor([s.last_token for s in seqs], dtype=torch.int64, device=device)
    history = torch.empty(steps, BATCH, dtype=torch.int64, device=device)
    sampler = ClockSampler(local) if rank == 0 else None
    launches_before = _lib.launches
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile_range:
        torch.cuda.profiler.start()
    # one packed int32 record per step, resident on the device; only the token ids are
    # filled in at run time (they come from the previous step's arg-max)
    width = bt.size(1)
    packed_all = torch.cat([torch.zeros(steps, BATCH, dtype=torch.int32, device=device), pos_all.int(), slot_all,
                            len_all, bt.flatten().expand(steps, -1)], dim=1).contiguous()
    with torch.inference_mode():
        ev0.record()
        for i in range(steps):
            packed_all[i, :BATCH] = ids
            bucket = graphs.stage_packed(packed_all[i], BATCH, width)
            graphs.run_graph(1, bucket)
            hidden = graphs.families[1].buffers['outputs'][:BATCH]
            ids = model.compute_logits(hidden).argmax(dim=-1)
            history[i] = ids
        ev1.record()
    barrier()
    if args.profile_range:
        torch.cuda.profiler.stop()
    ms_value = max_over_ranks(ev0.elapsed_time(ev1))
    launches = _lib.launches - launches_before
    clocks = sampler.stop() if sampler else None
    # The e2e loops below decode the same positions again (same context lengths, same bytes):
    # the sequences keep their length and the cache entries of the timed steps are rewritten.
    start_tokens = [list(s.token_ids) for s in seqs]

    def rewind():
        for s, toks in zip(seqs, start_tokens):
            s.token_ids = list(toks)

    # ---- e2e: K more steps through the public host API
    h2d = BATCH * 4 * 4 + BATCH * len(seqs[0].block_table) * 4          # one packed int32 record per step
    d2h = BATCH * 8
    barrier()
    ev0.record()
    e2e_steps(steps)
    ev1.record()
    barrier()
    ms_e2e_sync = max_over_ranks(ev0.elapsed_time(ev1))      # ModelRunner.run: host round trip every step
    rewind()
    barrier()
    ev0.record()
    runner.run_steps(seqs, steps)                            # multi-step decoding: one host sync per call
    ev1.record()
    barrier()
    ms_e2e = max_over_ranks(ev0.elapsed_time(ev1))

    # ---- one 16-position verify pass (graph, M = 16)
    drafts = [[int(t) for t in torch.randint(0, cfg.vocab_size, (VERIFY_M - 1,), generator=g)] for _ in seqs]
    runner.verify(seqs, drafts)
    barrier()
    ev0.record()
    runner.verify(seqs, drafts)
    ev1.record()
    barrier()
    ms_verify = max_over_ranks(ev0.elapsed_time(ev1))

    # ---- roofline of the dominant kernel: every W4A16 launch of one decode step, on the model's own
    # weights (3.3 GB, so nothing is served from L2), replayed as a graph of exactly those launches
    lins = [m for m in model.modules() if hasattr(m, "packed")]
    xin = {}
    for m in lins:
        xin.setdefault(m.in_features, torch.randn(BATCH, m.in_features, device=device, dtype=torch.float16))
    alg_bytes = sum(m.packed.numel() * 4 + m.scales.numel() * 2 + (m.zeros.numel() * 2 if m.zeros.numel() > 1 else 4)
                    + 2 * BATCH * (m.in_features + m.out_features) for m in lins)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side), torch.inference_mode():
        for m in lins:
            m(xin[m.in_features])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for m in lins:
                m(xin[m.in_features])
        reps = 5
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(side)
        for _ in range(reps):
            graph.replay()
        b.record(side)
        torch.cuda.synchronize()
        ms_lin = a.elapsed_time(b) / reps
    peaks, which = measured_peaks()
    achieved = alg_bytes / (ms_lin * 1e-3) / 1e9
    # DRAM traffic per launch from the ncu capture of this kernel at gate_up geometry, M = 32
    # (dram__bytes_read.sum + dram__bytes_write.sum = 52.3 MB for 53.74 MB of algorithmic bytes; the
    # output stays in L2), scaled to the mean launch of this graph by its algorithmic bytes.
    traffic = alg_bytes / len(lins) * (52.3 / 53.74)
    roofline = {"bound": "hbm", "kernel": f"w4a16_umma_kernel (M={BATCH}, all {len(lins)} W4A16 launches of one decode step)",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "of": which, "traffic": round(traffic),
                "bytes_per_launch": round(alg_bytes / len(lins)), "us_per_launch": round(ms_lin * 1e3 / len(lins), 2)}

    def teardown():
        # every rank: graphs (they hold NCCL kernels) first, then the process group; if the
        # teardown blocks all the same, leave without it once the result is out
        if world > 1:
            import threading
            guard = threading.Timer(30.0, os._exit, (0,))
            guard.daemon = True
            guard.start()
            runner.shutdown()
            parallel.shutdown()
            guard.cancel()

    if rank != 0:
        teardown()
        return
    tokens = BATCH * steps
    line = {
        "metric": METRIC, "value": round(tokens / (ms_value * 1e-3), 1), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(ms_value / steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": workload_config(world),
        "e2e": {"value": round(tokens / (ms_e2e * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e / steps, 4),
                "api": "ModelRunner.run_steps (multi-step decoding: per step one H2D record and one D2H token "
                       "copy, one host synchronisation per call)",
                "per_step_sync": {"value": round(tokens / (ms_e2e_sync * 1e-3), 1),
                                  "ms_per_step": round(ms_e2e_sync / steps, 4), "api": "ModelRunner.run"}},
        "gpu_launches": launches,
        "clocks": clocks,
        "roofline": roofline,
        "verify_pass_ms": round(ms_verify, 3),
        "setup_s": {"build": round(t_build, 1), "prefill": round(t_prefill, 1)},
        "context_tokens": len(seqs[0]),
    }
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        value, _, sample = cpu_tokens_per_s(cfg, PROMPT + 256, 3, 1, threads)
        line["cpu_baseline"] = {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": sample + "; 3 timed samples"}
    print(json.dumps(line), flush=True)
    teardown()


def run_case(args):
    """One small single-kernel case (inputs larger than L2, a few launches): the command that the
    `ncu --set full` captures summarised under profiles/ run.  Prints one JSON line with the CUDA-event
    time per launch (graph replay over distinct inputs, so nothing is served from L2)."""
    import torch
    from linkq2_b200.kernels.gemlite.ops import set_constant_weights
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    from linkq2_b200.runtime.backends import make_quant_linear

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device; the operators have no CPU path")
    torch.cuda.set_device(0)
    g = torch.Generator().manual_seed(0)
    peaks, which = measured_peaks()
    if args.case in ("w4a16_gemv", "w4a16_m32"):
        k, n, m, copies = 4096, 24576, (1 if args.case == "w4a16_gemv" else 32), 4
        vals = (torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8).to(torch.int16) - 8).to(torch.int8)
        scale = (torch.rand(n, k // 128, generator=g) * 0.01 + 0.001).half()
        layers = [make_quant_linear("b200", vals, scale, group_size=128, symmetric=True, device="cuda",
                                    dtype=torch.float16) for _ in range(copies)]
        x = torch.randn(m, k, device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        set_constant_weights(True)                     # as the runtime does once the checkpoint is loaded
        calls = [lambda l=l: l(x) for l in layers]
        nbytes = k * n // 2 + 2 * (k // 128) * n + 2 * m * (k + n)
        what = f"gate_up geometry K={k} N={n} M={m}, {copies} distinct weight copies"
    else:
        hq, hkv, d, page, bs, ctx = 32, 8, 128, 256, 64, 4096
        nb = bs * (ctx // page)
        slots = nb * page
        kq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
        vq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
        ks = (torch.rand(hkv, d, device="cuda") * 0.1 + 0.05).half()
        vs = (torch.rand(slots, hkv, 2, device="cuda") * 0.1 + 0.05).half()
        table = torch.randperm(nb, generator=g).int().view(bs, -1).cuda()
        q = (torch.randn(bs, hq, d, device="cuda") * 0.5).half()
        lens = torch.full((bs,), ctx, dtype=torch.int32, device="cuda")
        calls = [lambda: paged_attention_decode(q, (kq, ks), (vq, vs), table, lens, block_n=page,
                                                num_kv_heads=hkv)] * 3
        nbytes = bs * ctx * hkv * (d + 2 * (d // 64)) + 4 * bs * hq * d
        what = f"decode batch {bs}, context {ctx}, Qwen3-8B heads, page {page}, v_group 64 (277 MB of cache)"
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
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(5):
            a.record(side)
            graph.replay()
            b.record(side)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
    us = sorted(times)[len(times) // 2] * 1e3 / len(calls)
    gbs = nbytes / us / 1e3
    print(json.dumps({"case": args.case, "workload": what, "launches_timed": len(calls), "replays": "median of 5",
                      "us_per_launch": round(us, 2), "algorithmic_bytes_per_launch": nbytes,
                      "achieved_gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 4), "of": which}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed decode steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--case", default=None, choices=["w4a16_gemv", "w4a16_m32", "kv4_decode"],
                    help="run one small single-kernel case instead of the workload (the profiled cases)")
    args = ap.parse_args()
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
