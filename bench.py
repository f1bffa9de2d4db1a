"""Qwen3-8B W4 + KV4 batched decode throughput on N B200s (tensor parallel), with
the W4A16 kernel's HBM roofline and the CPU restatement timed beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config qwen3_8b|qwen3_1p7b]

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
class Geometry:
    """Qwen3-8B shapes of the workload, spelled out here so that the CPU arm imports
    nothing of the GPU package."""
    hidden_size, intermediate_size, num_hidden_layers = 4096, 12288, 36
    num_attention_heads, num_key_value_heads, head_dim, vocab_size = 32, 8, 128, 151936


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


def cpu_tokens_per_s(cfg, context, steps, warmup, threads, budget_s=150.0):
    """``steps`` timed samples (fewer if ``budget_s`` of wall time runs out first).  Every
    sample times a part of a step and scales it up, which the returned description and the
    ``sampling`` factors state: the whole step is never executed on the CPU."""
    import torch
    sampled = 2
    layer = cpu_step_sample(cfg, sampled, context, threads)
    g = torch.Generator().manual_seed(1)
    head = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * 0.02)
    xh = torch.randn(BATCH, cfg.hidden_size, generator=g)
    for _ in range(max(1, warmup)):
        layer()
    times = []
    started = time.perf_counter()
    for _ in range(steps):
        if times and time.perf_counter() - started > budget_s:
            break
        lin, att = layer()
        t0 = time.perf_counter()
        (xh @ head.t()).argmax(-1)
        th = time.perf_counter() - t0
        times.append(cfg.num_hidden_layers * (lin + att) + th)
    step = sum(times) / len(times)
    sample = (f"per step: 1 of {cfg.num_hidden_layers} decoder layers (7 dense fp32 projections at M={BATCH}, "
              f"KV4 store+decode for {sampled} of {BATCH} sequences at context {context}, scaled x{BATCH // sampled}) "
              f"+ fp32 LM head; step time = {cfg.num_hidden_layers} x layer + head")
    sampling = {"layers_timed": 1, "layers_total": cfg.num_hidden_layers, "sequences_timed": sampled,
                "sequences_total": BATCH, "samples": len(times)}
    return BATCH / step, step * 1e3, sample, sampling


def run_reference(args):
    """The reference's CPU arithmetic for the workload on the host cores (the oracle port: the
    reference's own runtime is CUDA-only).  Rank 0 alone works.  ``ms_per_step`` is an
    extrapolated step time - one decoder layer and two of the 32 sequences are timed per
    sample and scaled - and the line says so."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = Geometry
    threads = os.cpu_count() or 1
    steps, warmup = max(1, args.steps), max(1, args.warmup)
    value, ms, sample, sampling = cpu_tokens_per_s(cfg, PROMPT + 256, steps, warmup, threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": sampling["samples"], "warmup": warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.gpus),
        "extrapolated": True, "sampling": sampling,
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + f"; {sampling['samples']} timed samples"},
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
        """``index`` is the CUDA device index of this process; nvidia-smi counts physical
        GPUs and ignores CUDA_VISIBLE_DEVICES, so the device is named by its UUID."""
        self.proc = None
        try:
            import torch
            target = "GPU-" + str(torch.cuda.get_device_properties(index).uuid)
        except Exception:
            target = str(index)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", target], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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


def graph_us_per_call(calls, min_ms=100.0):
    """Device time per call in microseconds: the calls are captured into one CUDA graph on a
    side stream and the graph is replayed back to back for at least ``min_ms`` between two CUDA
    events recorded on that stream.  The callers pass calls over distinct inputs whose total
    exceeds the 126 MB L2, so nothing is served from cache between replays."""
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
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(3):
            graph.replay()
        a.record(side)
        graph.replay()
        b.record(side)
        torch.cuda.synchronize()
        reps = max(3, int(min_ms / max(a.elapsed_time(b), 1e-3)) + 1)
        a.record(side)
        for _ in range(reps):
            graph.replay()
        b.record(side)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
    return ms * 1e3 / (reps * len(calls)), {"replays": reps, "timed_ms": round(ms, 2), "calls_per_replay": len(calls)}


def roofline_entry(kernel, nbytes, us, peaks, which, traffic, extra):
    gbs = nbytes / us / 1e3
    return {"bound": "hbm", "kernel": kernel, "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(gbs / peaks["hbm_gbs"], 4), "of": which, "frac_of_nominal_8tbs": round(gbs / 8000.0, 4),
            "traffic": traffic, "bytes_per_launch": round(nbytes), "us_per_launch": round(us, 2), **extra}


def roofline_gemv_config1(peaks, which):
    """Configuration 1: K = N = 4096, M = 1, asymmetric uint4 group 128 (fp16 scale and zero
    point per group): 8 929 280 algorithmic bytes per launch.  24 distinct weight copies
    (214 MB) rotate through the graph."""
    import torch
    from linkq2_b200.runtime.backends import make_quant_linear
    k = n = 4096
    g = torch.Generator().manual_seed(1)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    scale = (torch.rand(n, k // 128, generator=g) * 0.004 + 0.001).half()
    zero = torch.randint(0, 16, (n, k // 128), generator=g).half()
    layers = [make_quant_linear("b200", codes, scale, group_size=128, symmetric=False, zero_point=zero,
                                device="cuda", dtype=torch.float16) for _ in range(24)]
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    nbytes = k * n // 2 + 2 * 2 * (k // 128) * n + 2 * (k + n)
    assert nbytes == 8929280
    us, how = graph_us_per_call([lambda l=l: l(x) for l in layers])
    # ncu capture of this kernel (gate_up geometry, M = 1): DRAM read + write = 53.6 MB for 53.5 MB
    # algorithmic, i.e. traffic = algorithmic bytes; scaled here by the bytes of this shape
    return roofline_entry("w4a16_stream_kernel (configs[0]: 4096x4096, M=1, affine g128; 24 rotating weight copies)",
                          nbytes, us, peaks, which, round(nbytes * 53.6 / 53.5), how)


def roofline_kv4_config3(peaks, which):
    """Configuration 3 at batch 64: contexts drawn uniformly from 512..32768 (seeded), blocks
    randomly permuted, Qwen3-8B heads, page 256, v_group 64; 1056 bytes per cached token plus
    queries and outputs.  The pool holds random bits: the kernel's time does not depend on the
    values (the parity tests cover this configuration with real quantized data)."""
    import torch
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    hq, hkv, d, page, bs = 32, 8, 128, 256, 64
    g = torch.Generator().manual_seed(3)
    lens = torch.randint(512, 32769, (bs,), generator=g)
    blocks = [(int(l) + page - 1) // page for l in lens]
    nb = sum(blocks)
    perm = torch.randperm(nb, generator=g).int()
    table = torch.full((bs, max(blocks)), -1, dtype=torch.int32)
    at = 0
    for i, n in enumerate(blocks):
        table[i, :n] = perm[at:at + n]
        at += n
    slots = nb * page
    kq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
    vq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
    ks = (torch.rand(hkv, d, device="cuda") * 0.1 + 0.05).half()
    vs = (torch.rand(slots, hkv, 2, device="cuda") * 0.1 + 0.05).half()
    q = (torch.randn(bs, hq, d, device="cuda") * 0.5).half()
    table, lens_d = table.cuda(), lens.int().cuda()
    total = int(lens.sum())
    nbytes = total * hkv * (d + 2 * (d // 64)) + 4 * bs * hq * d
    us, how = graph_us_per_call([lambda: paged_attention_decode(q, (kq, ks), (vq, vs), table, lens_d, block_n=page,
                                                                num_kv_heads=hkv)] * 2)
    # ncu capture (batch 64 x 4096): DRAM read + write 279.6 MB for 277.9 MB algorithmic
    return roofline_entry(f"kv4_decode_fast_kernel (configs[2]: batch 64, contexts U(512..32768) seed 3, {total} cached tokens)",
                          nbytes, us, peaks, which, round(nbytes * 279.6 / 277.9), how)


def self_check(tp, device):
    """Correctness evidence in the bench line at every rank count: a seeded 2-layer checkpoint
    (8 query / 8 KV heads, so it shards over up to 8 ranks) is loaded through the same
    tensor-parallel split, CUDA graphs and exchange kernels as the workload and decoded greedily;
    the tokens must equal the fixture ``tests/golden/tp_parity.npz`` (produced by the CPU oracle
    model; this function only reads the file)."""
    import tempfile
    import numpy as np
    import torch
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig
    from linkq2_b200.runtime.model.qwen3 import ModelConfig
    from linkq2_b200.runtime.quantization import build_from_checkpoint, save_random_checkpoint
    from linkq2_b200.runtime.state import BlockPool, Sequence
    fixture = ROOT / "tests" / "golden" / "tp_parity.npz"
    if not fixture.exists():
        return {"tokens_equal": None, "error": "tests/golden/tp_parity.npz is missing"}
    gold = np.load(fixture)
    cfg = ModelConfig.from_dict(json.loads(bytes(gold["config"]).decode()))
    seed, new_tokens, cases = (int(v) for v in gold["meta"])
    with tempfile.TemporaryDirectory() as tmp:
        path = save_random_checkpoint(Path(tmp) / "w4", cfg, seed=seed)
        model = build_from_checkpoint(path, device=device, max_position=1024)
    rc = RunnerConfig(kvcache_block_size=128, num_kvcache_blocks=16, max_num_seqs=4, max_model_len=512,
                      enforce_eager=False)
    shape = (cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim)
    runner = ModelRunner(model, rc, device=device, smooth_kv={"lambda": torch.ones(shape),
                                                              "kscale": torch.full(shape, float(gold["kscale"][0]))})
    prompts = [[int(t) for t in gold[f"prompt{i}"]] for i in range(cases)]
    seqs = [Sequence(p, 128) for p in prompts]
    pool = BlockPool(16, shuffle_seed=5)
    for s in seqs:
        pool.ensure(s, len(s) + new_tokens + 1)
    first = runner.run(seqs, True)
    out = [[t] for t in first]
    for s, t in zip(seqs, first):
        s.append(t)
    for i in range(new_tokens - 1):
        runner.keep_logits = i == new_tokens - 2          # the tokens come from the pair exchange; the last
        step = runner.run(seqs, False)                    # step also gathers the logits for the comparison
        for s, o, t in zip(seqs, out, step):
            s.append(t)
            o.append(t)
    logits = runner.last_logits.float().cpu()
    want = [[int(t) for t in gold[f"tokens{i}"]] for i in range(cases)]
    err = max(float((logits[i] - torch.from_numpy(gold[f"logits{i}"])).abs().max()
                    / torch.from_numpy(gold[f"logits{i}"]).pow(2).mean().sqrt()) for i in range(cases))
    timeouts = tp.exchange.timeouts() if tp.exchange is not None else 0
    replays = runner.graph_replays
    runner.shutdown()
    return {"tokens_equal": out == want, "sequences": cases, "tokens_per_sequence": new_tokens,
            "final_logits_err_over_rms": round(err, 5), "graph_replays": replays,
            "allreduce_timeouts": int(timeouts), "exchange": "peer" if tp.exchange is not None else
            ("nccl" if tp.size > 1 else "none"),
            "against": "tests/golden/tp_parity.npz (CPU oracle model on the same seeded checkpoint)"}


def run_b200(args):
    import torch
    import torch.distributed as dist
    from linkq2_b200 import _lib
    from linkq2_b200.runtime import parallel
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig, amax_calibration
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

    small = args.config == "qwen3_1p7b"
    cfg = ModelConfig.qwen3_1p7b() if small else ModelConfig.qwen3_8b()
    batch, prompt_len = (1, 512) if small else (BATCH, PROMPT)
    if small and world != 1:
        raise SystemExit("configs[3] (Qwen3-1.7B, batch 1) is a single-GPU configuration")
    steps, warmup = args.steps, max(args.warmup, 3)
    max_len = prompt_len + warmup + steps + VERIFY_M + 8
    max_len = (max_len + 255) // 256 * 256
    page = 256
    blocks_per_seq = max_len // page
    rc = RunnerConfig(kvcache_block_size=page, num_kvcache_blocks=batch * blocks_per_seq + 4, v_group=64,
                      max_num_seqs=batch, max_model_len=max_len, enforce_eager=False,
                      spec_num_drafts=VERIFY_M - 1)
    t_build = time.time()
    model = build_random(cfg, seed=0, group_size=128, device=device, max_position=max_len + 64)
    runner = ModelRunner(model, rc, device=device,
                         smooth_kv=amax_calibration(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim, 0.5))
    torch.cuda.synchronize()
    t_build = time.time() - t_build

    # ---- prompts and chunked prefill (untimed for the metric; its own rate is reported)
    g = torch.Generator().manual_seed(1234)
    pool = BlockPool(rc.num_kvcache_blocks, shuffle_seed=7)
    seqs = []
    for _ in range(batch):
        s = Sequence(torch.randint(0, cfg.vocab_size, (prompt_len,), generator=g).tolist(), page)
        pool.ensure(s, max_len)
        seqs.append(s)
    chunk = prompt_len if small else CHUNK
    torch.cuda.synchronize()
    t_prefill = time.time()
    first = None
    for start in range(0, prompt_len, chunk):
        first = runner.run(seqs, True, counts=[chunk] * batch)
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
    pos_all = torch.tensor([[base_len - 1 + i] * batch for i in range(steps)], dtype=torch.int64, device=device)
    slot_all = torch.tensor([[s.slot(base_len - 1 + i) for s in seqs] for i in range(steps)],
                            dtype=torch.int32, device=device)
    len_all = torch.tensor([[base_len + i] * batch for i in range(steps)], dtype=torch.int32, device=device)
    ids = torch.tensor([s.last_token for s in seqs], dtype=torch.int64, device=device)
    history = torch.empty(steps, batch, dtype=torch.int64, device=device)
    sampler = ClockSampler(local) if rank == 0 else None
    launches_before = _lib.launches
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile_range:
        torch.cuda.profiler.start()
    # one packed int32 record per step, resident on the device; only the token ids are
    # filled in at run time (they come from the previous step's arg-max)
    width = bt.size(1)
    packed_all = torch.cat([torch.zeros(steps, batch, dtype=torch.int32, device=device), pos_all.int(), slot_all,
                            len_all, bt.flatten().expand(steps, -1)], dim=1).contiguous()
    with torch.inference_mode():
        ev0.record()
        for i in range(steps):
            packed_all[i, :batch] = ids
            bucket = graphs.stage_packed(packed_all[i], batch, width)
            graphs.run_graph(1, bucket)
            hidden = graphs.families[1].buffers['outputs'][:batch]
            ids = model.greedy_tokens(hidden)          # arg-max; a (value, index) exchange under tensor parallelism
            history[i] = ids
        ev1.record()
    barrier()
    if args.profile_range:
        torch.cuda.profiler.stop()
    ms_value = max_over_ranks(ev0.elapsed_time(ev1))
    launches = _lib.launches - launches_before
    # The e2e loops below decode the same positions again (same context lengths, same bytes):
    # the sequences keep their length and the cache entries of the timed steps are rewritten.
    start_tokens = [list(s.token_ids) for s in seqs]

    def rewind():
        for s, toks in zip(seqs, start_tokens):
            s.token_ids = list(toks)

    # ---- e2e: K more steps through the public host API
    h2d = batch * 4 * 4 + batch * len(seqs[0].block_table) * 4          # one packed int32 record per step
    d2h = batch * 8
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
    clocks = sampler.stop() if sampler else None

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
    # weights (3.3 GB at Qwen3-8B size, so nothing is served from L2), replayed as a graph of exactly
    # those launches for at least 100 ms
    peaks, which = measured_peaks()
    lins = [m for m in model.modules() if hasattr(m, "packed")]

    def lin_bytes(rows):
        return sum(m.packed.numel() * 4 + m.scales.numel() * 2 + (m.zeros.numel() * 2 if m.zeros.numel() > 1 else 4)
                   + 2 * rows * (m.in_features + m.out_features) for m in lins)

    def lin_calls(rows):
        xin = {}
        for m in lins:
            xin.setdefault(m.in_features, torch.randn(rows, m.in_features, device=device, dtype=torch.float16))
        return [lambda m=m: m(xin[m.in_features]) for m in lins]

    alg_bytes = lin_bytes(batch)
    us_lin, how = graph_us_per_call(lin_calls(batch))
    # DRAM traffic per launch from the ncu capture of this kernel at gate_up geometry, M = 32
    # (dram__bytes_read.sum + dram__bytes_write.sum = 52.3 MB for 53.74 MB of algorithmic bytes; the
    # output stays in L2), scaled to the mean launch of this graph by its algorithmic bytes.
    kernel = "w4a16_stream_kernel" if batch <= 8 else "w4a16_umma_kernel"
    roofline = roofline_entry(f"{kernel} (M={batch}, all {len(lins)} W4A16 launches of one decode step)",
                              alg_bytes / len(lins), us_lin, peaks, which,
                              round(alg_bytes / len(lins) * (52.3 / 53.74)), how)

    # ---- where the verify pass goes: the M = batch * 16 projections and the verify attention
    verify_parts = None
    if not small:
        rows = batch * VERIFY_M
        us_vlin, _ = graph_us_per_call(lin_calls(rows), min_ms=30.0)
        attn = next(m for m in model.modules() if hasattr(m, "k_cache") and m.k_cache is not None)
        from linkq2_b200.kernels.kv4 import paged_attention_decode
        hq, hkv, d = cfg.num_attention_heads // world, cfg.num_key_value_heads // world, cfg.head_dim
        qv = torch.randn(rows, hq, d, device=device, dtype=torch.float16)
        lens_v = torch.tensor([len(s) for s in seqs], dtype=torch.int32, device=device)
        us_vattn, _ = graph_us_per_call(
            [lambda: paged_attention_decode(qv, attn.k_cache, attn.v_cache, bt, lens_v, block_n=page, num_kv_heads=hkv,
                                            v_group=64, verify_m=VERIFY_M)], min_ms=30.0)
        flops = sum(2 * rows * m.in_features * m.packed.shape[1] for m in lins)
        verify_parts = {"linears_ms": round(us_vlin * len(lins) / 1e3, 3),
                        "linears_tflops": round(flops / (us_vlin * len(lins)) / 1e6, 1),
                        "attention_ms": round(us_vattn * cfg.num_hidden_layers / 1e3, 3),
                        "attention_us_per_layer": round(us_vattn, 1), "rows": rows,
                        "note": "kernels timed alone (graph replay); the pass also holds the norms, the fused "
                                "pre-attention kernels, the exchange under tensor parallelism and the LM head"}

    extra = {}
    if world == 1 and not small and not args.no_kernel_rooflines:
        extra["roofline_gemv"] = roofline_gemv_config1(peaks, which)
        extra["roofline_kv4"] = roofline_kv4_config3(peaks, which)
    if small:
        # batch-1 decode is the weight-streaming kernel inside a model
        extra["tpot_ms"] = round(ms_value / steps, 4)
        extra["reference_published"] = "8.9 ms TPOT for the 8B model on an RTX 4090 D (benchmarks/runtime/engine/RESULTS.md:11-12)"

    timeouts_main = tp.exchange.timeouts() if tp.exchange is not None else 0
    runner.shutdown()
    del runner
    torch.cuda.empty_cache()
    try:
        check = self_check(tp, device)
    except Exception as e:                                  # the line must still come out
        check = {"tokens_equal": None, "error": f"{type(e).__name__}: {e}"[:500]}
    check["allreduce_timeouts"] = int(check.get("allreduce_timeouts", 0)) + int(timeouts_main)

    def teardown():
        # every rank: graphs (they hold NCCL kernels) first, then the process group; if the
        # teardown blocks all the same, leave without it once the result is out
        if world > 1:
            import threading
            guard = threading.Timer(30.0, os._exit, (0,))
            guard.daemon = True
            guard.start()
            parallel.shutdown()
            guard.cancel()

    if rank != 0:
        teardown()
        return
    tokens = batch * steps
    line = {
        "metric": METRIC if not small else "qwen3_1p7b_w4_kv4_decode_tokens_per_s",
        "value": round(tokens / (ms_value * 1e-3), 1), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(ms_value / steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": workload_config(world) if not small else workload_config_small(),
        "e2e": {"value": round(tokens / (ms_e2e * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e / steps, 4),
                "api": "ModelRunner.run_steps (multi-step decoding: per step one H2D record and one D2H token "
                       "copy, one host synchronisation per call)",
                "per_step_sync": {"value": round(tokens / (ms_e2e_sync * 1e-3), 1),
                                  "ms_per_step": round(ms_e2e_sync / steps, 4), "api": "ModelRunner.run"}},
        "gpu_launches": launches,
        "clocks": clocks,
        "roofline": roofline,
        **extra,
        "verify_pass_ms": round(ms_verify, 3),
        "verify_parts": verify_parts,
        "parity_check": check,
        "setup_s": {"build": round(t_build, 1), "prefill": round(t_prefill, 1)},
        "prefill_tokens_per_s": round(batch * prompt_len / t_prefill, 1),
        "context_tokens": len(seqs[0]),
    }
    if world == 1 and not args.no_cpu_baseline and not small:
        threads = os.cpu_count() or 1
        value, _, sample, sampling = cpu_tokens_per_s(Geometry, PROMPT + 256, 3, 1, threads)
        line["cpu_baseline"] = {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": sample + "; 3 timed samples", "extrapolated": True, "sampling": sampling}
    print(json.dumps(line), flush=True)
    teardown()


def workload_config_small():
    return {"workload": "configs[3]: Qwen3-1.7B geometry (28 layers, hidden 2048, inter 6144, 16 q / 8 kv heads, "
                        "head_dim 128, vocab 151936, tied head), random init RTN-W4 g128 + KV4 (page 256, v_group 64)",
            "batch": 1, "prompt_tokens": 512, "prefill": "one 512-token step (untimed)",
            "step": "one decode forward: 1 sequence x 1 new token, CUDA graph + fp16 LM head + argmax",
            "parallelism": "tp1", "l2": "per-step working set (0.7 GB weights + 0.6 GB head) exceeds the 126 MB L2"}


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
    flops = None
    if args.case in ("w4a16_gemv", "w4a16_m32", "w4a16_m512"):
        k, n, m, copies = 4096, 24576, {"w4a16_gemv": 1, "w4a16_m32": 32, "w4a16_m512": 512}[args.case], 4
        vals = (torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8).to(torch.int16) - 8).to(torch.int8)
        scale = (torch.rand(n, k // 128, generator=g) * 0.01 + 0.001).half()
        layers = [make_quant_linear("b200", vals, scale, group_size=128, symmetric=True, device="cuda",
                                    dtype=torch.float16) for _ in range(copies)]
        x = torch.randn(m, k, device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        set_constant_weights(True)                     # as the runtime does once the checkpoint is loaded
        calls = [lambda l=l: l(x) for l in layers]
        nbytes = k * n // 2 + 2 * (k // 128) * n + 2 * m * (k + n)
        flops = 2.0 * m * k * n if m >= 256 else None          # tensor-bound from a few hundred rows on
        what = f"gate_up geometry K={k} N={n} M={m}, {copies} distinct weight copies"
    elif args.case == "kv4_verify":
        hq, hkv, d, page, bs, ctx, mrows = 32, 8, 128, 256, 32, 2200, 16
        nb = bs * ((ctx + mrows + page - 1) // page)
        slots = nb * page
        kq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
        vq = torch.randint(-2**31, 2**31 - 1, (slots, hkv, d // 8), dtype=torch.int32, device="cuda")
        ks = (torch.rand(hkv, d, device="cuda") * 0.1 + 0.05).half()
        vs = (torch.rand(slots, hkv, 2, device="cuda") * 0.1 + 0.05).half()
        table = torch.randperm(nb, generator=g).int().view(bs, -1).cuda()
        q = (torch.randn(bs * mrows, hq, d, device="cuda") * 0.5).half()
        lens = torch.full((bs,), ctx, dtype=torch.int32, device="cuda")
        calls = [lambda: paged_attention_decode(q, (kq, ks), (vq, vs), table, lens, block_n=page,
                                                num_kv_heads=hkv, verify_m=mrows)] * 3
        nbytes = bs * (ctx + mrows - 1) * hkv * (d + 2 * (d // 64)) + 4 * bs * mrows * hq * d
        # QK^T and PV over the cached tokens, 64 query rows per KV head, without the second pass that the
        # fp16-split queries add to QK^T
        flops = 4.0 * bs * hq * mrows * (ctx + mrows - 1) * d
        what = (f"verify: batch {bs}, context {ctx}, {mrows} positions, Qwen3-8B heads, page {page}, v_group 64 "
                f"({bs * ctx * hkv * 132 // 2**20} MB of cache; bound by the warp-level tensor op, see achieved_tflops)")
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
    line = {"case": args.case, "workload": what, "launches_timed": len(calls), "replays": "median of 5",
            "us_per_launch": round(us, 2), "algorithmic_bytes_per_launch": nbytes,
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 4), "of": which}
    if flops is not None:
        line["achieved_tflops"] = round(flops / us / 1e6, 1)
        line["frac_of_bf16_burst"] = round(flops / us / 1e6 / peaks["bf16_tflops"], 4)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-rooflines", action="store_true",
                    help="skip the single-kernel roofline_gemv / roofline_kv4 records of the N=1 line")
    ap.add_argument("--config", default="qwen3_8b", choices=["qwen3_8b", "qwen3_1p7b"],
                    help="qwen3_8b: the workload of the metric (configs[4]); qwen3_1p7b: configs[3], batch-1 decode")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed decode steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--case", default=None, choices=["w4a16_gemv", "w4a16_m32", "w4a16_m512", "kv4_decode", "kv4_verify"],
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
