"""Tensor-parallel decoding on two GPUs (one process per GPU, NCCL): greedy tokens
of the sharded model — column-split q/k/v/gate/up, row-split o/down with an
all-reduce captured in each rank's CUDA graph, KV heads split — must equal the
single-sequence CPU oracle, exactly as the one-GPU runtime's do.  Skipped on a
box with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HQ, HKV, NEW_TOKENS = 4, 2, 32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ckpt, prompts, eager, results):
    from linkq2_b200.runtime import parallel
    from linkq2_b200.runtime.execute.model_runner import ModelRunner, RunnerConfig, amax_calibration
    from linkq2_b200.runtime.quantization import build_from_checkpoint
    from tests.test_runtime_gpu import generate
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    tp = parallel.init_from_env("nccl")
    device = f"cuda:{rank}"
    model = build_from_checkpoint(ckpt, device=device, max_position=512)
    rc = RunnerConfig(kvcache_block_size=128, num_kvcache_blocks=16, max_num_seqs=4, max_model_len=512,
                      enforce_eager=eager, spec_num_drafts=0)
    runner = ModelRunner(model, rc, smooth_kv=amax_calibration(2, HKV, 64, 0.3), device=device)
    runner.keep_logits = True
    tokens, _ = generate(runner, prompts, NEW_TOKENS, 16)
    # the pair exchange of the greedy path against the arg-max of the gathered logits, ties included
    g = torch.Generator(device=device).manual_seed(3)
    h = torch.randn(6, model.config.hidden_size, generator=g, device=device).half()
    h[4] = 0                                    # every logit equal: the lowest index must win
    h[5] = h[3]
    assert torch.equal(model.greedy_tokens(h), model.compute_logits(h).argmax(dim=-1))
    results[rank] = (tokens, runner.last_logits.float().cpu(), runner.graph_replays, tp.size)
    runner.shutdown()                       # graphs hold NCCL kernels: release them before the group
    parallel.shutdown()


def _exchange_worker(rank, world, port, results):
    """The library's peer-memory all-reduce against a rank-ordered fp32 sum of the
    all-gathered addends (bit-exact), eagerly and replayed from a CUDA graph."""
    import torch.distributed as dist
    from linkq2_b200.runtime import parallel
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    tp = parallel.init_from_env("nccl")
    if tp.exchange is None:
        results[rank] = "unavailable"
        parallel.shutdown()
        return
    g = torch.Generator().manual_seed(100 + rank)

    def expected_sum(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        acc = torch.zeros_like(x, dtype=torch.float32)
        for part in parts:                      # rank order, fp32, one rounding at the end
            acc += part.float()
        return acc.half()

    checked = 0
    for shape in [(1, 4096), (32, 4096), (3, 8), (512, 1024), (17, 2048), (32, 4096)]:
        for _ in range(3):                      # consecutive calls alternate the buffer halves
            x = (torch.randn(*shape, generator=g) * (1 + rank)).half().cuda()
            want = expected_sum(x)
            assert tp.exchange.accepts(x)
            got = tp.all_reduce(x.clone())
            torch.cuda.synchronize()
            assert torch.equal(got, want), (shape, (got.float() - want.float()).abs().max())
            checked += 1
    # the same exchange inside the residual RMSNorm kernel
    from linkq2_b200.kernels.fused import rmsnorm, rmsnorm_allreduce
    for rows, hidden in [(1, 4096), (32, 4096), (5, 1024), (64, 8192), (32, 4096)]:
        for _ in range(2):
            x = (torch.randn(rows, hidden, generator=g) * (1 + rank)).half().cuda()
            res = torch.randn(rows, hidden, generator=torch.Generator().manual_seed(rows + hidden)).half().cuda()
            w = (1 + 0.1 * torch.randn(hidden, generator=torch.Generator().manual_seed(hidden))).half().cuda()
            want_out, want_res = rmsnorm(expected_sum(x), w, 1e-6, res)
            got_out, got_res = rmsnorm_allreduce(x, w, 1e-6, res, tp.exchange)
            torch.cuda.synchronize()
            assert torch.equal(got_res, want_res) and torch.equal(got_out, want_out), (rows, hidden)
            checked += 1
    # the producer side fused into the projection: the kernel pushes, the norm only gathers
    from linkq2_b200.runtime.backends import make_quant_linear
    for rows, k, n in [(32, 512, 4096), (16, 1536, 4096), (64, 256, 1024), (9, 512, 4096)]:
        gw = torch.Generator().manual_seed(1000 * rank + k)
        vals = (torch.randint(0, 16, (n, k), generator=gw, dtype=torch.uint8).to(torch.int16) - 8).to(torch.int8)
        scale = (torch.rand(n, k // 128, generator=gw) * 0.01 + 0.001).half()
        layer = make_quant_linear("b200", vals, scale, group_size=128, symmetric=True, device="cuda",
                                  dtype=torch.float16)
        xin = torch.randn(rows, k, generator=g).half().cuda()
        res = torch.randn(rows, n, generator=torch.Generator().manual_seed(rows + n)).half().cuda()
        w = (1 + 0.1 * torch.randn(n, generator=torch.Generator().manual_seed(n))).half().cuda()
        for _ in range(2):
            want_out, want_res = rmsnorm_allreduce(layer(xin), w, 1e-6, res, tp.exchange)
            partial = layer.forward_push(xin, tp.exchange)
            got_out, got_res = rmsnorm_allreduce(partial, w, 1e-6, res, tp.exchange, pushed=True)
            torch.cuda.synchronize()
            assert torch.equal(partial, layer(xin))
            assert torch.equal(got_res, want_res) and torch.equal(got_out, want_out), (rows, k, n)
        checked += 1
    big = torch.ones(2048, 4096, dtype=torch.float16, device="cuda")           # above the limit: NCCL
    assert not tp.exchange.accepts(big)
    assert torch.equal(tp.all_reduce(big), torch.full_like(big, world))
    # a chain of dependent all-reduces inside a CUDA graph
    a = (torch.randn(32, 4096, generator=g)).half().cuda()
    side = torch.cuda.Stream()

    def chain():
        y = tp.all_reduce(a * 0.5)
        z = tp.all_reduce(y * 0.25 + a)
        return tp.all_reduce(z * 0.125)
    with torch.cuda.stream(side):
        eager = chain()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out = chain()
        for _ in range(4):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager)
    assert tp.exchange.timeouts() == 0
    del graph
    results[rank] = checked
    parallel.shutdown()


def test_peer_memory_all_reduce_is_bit_exact():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_exchange_worker, args=(world, port, results), nprocs=world, join=True)
        results = dict(results)
    if any(v == "unavailable" for v in results.values()):
        pytest.skip("CUDA IPC / peer access is not available between these GPUs")
    assert results == {0: 32, 1: 32}


@pytest.mark.parametrize("eager", [True, False])
def test_two_gpu_tokens_match_oracle(tmp_path, eager):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from linkq2_b200.runtime.model.qwen3 import ModelConfig
    from oracle import qwen3 as oq
    from tests.test_runtime_gpu import CFG, write_checkpoint
    weights = write_checkpoint(tmp_path / "w4", hq=HQ, hkv=HKV)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 127, (n,), generator=g).tolist() for n in (21, 34)]
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, port, str(tmp_path / "w4"), prompts, eager, results), nprocs=world, join=True)
        results = dict(results)
    assert set(results) == {0, 1}
    assert results[0][0] == results[1][0]                       # every rank decodes the same tokens
    assert results[0][3] == 2
    cfg = ModelConfig.from_dict(dict(CFG, num_attention_heads=HQ, num_key_value_heads=HKV))
    for i, prompt in enumerate(prompts):
        oracle = oq.OracleQwen3(cfg, weights, kscale=torch.full((2, HKV, 64), 0.3), max_tokens=512)
        assert results[0][0][i] == oracle.greedy(prompt, NEW_TOKENS, chunk=16)
        expected = oracle.last_logits[-1]
        for rank in (0, 1):
            assert (results[rank][1][i] - expected).abs().max() / expected.pow(2).mean().sqrt() < 2e-2
    if not eager:
        assert results[0][2] == NEW_TOKENS - 1
