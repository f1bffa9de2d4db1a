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
    tokens, _ = generate(runner, prompts, NEW_TOKENS, 16)
    results[rank] = (tokens, runner.last_logits.float().cpu(), runner.graph_replays, tp.size)
    runner.shutdown()                       # graphs hold NCCL kernels: release them before the group
    parallel.shutdown()


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
