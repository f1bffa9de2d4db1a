"""Tensor-parallel sharding of logical quantized tensors, checked on CPU with two
gloo ranks: column-split projections concatenate to the full output, row-split
projections sum to it through an all-reduce."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4a16 as ow


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    from linkq2_b200.runtime import parallel
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tp = parallel.init_from_env("gloo")
    assert (tp.rank, tp.size) == (rank, world)
    group = 128
    w_col, w_row = ow.seeded_weight(256, 512, 1), ow.seeded_weight(128, 1024, 2)
    x = ow.seeded_activation(3, 512, 3)
    for affine in (False, True):
        def quant(w):
            if affine:
                v, s, z = ow.affine_quantize(w, group)
                return {"values": v, "scale": s, "zero_point": z, "input_scale": torch.ones(w.shape[1]).half() * 2}
            v, s = ow.rtn_quantize(w, group)
            return {"values": v, "scale": s, "zero_point": None, "input_scale": None}

        def dense(d):
            out = ow.dequantize_fp32(d["values"], d["scale"], symmetric=not affine, zero_point=d["zero_point"],
                                     input_scale=d["input_scale"])
            return out
        full_c, full_r = quant(w_col), quant(w_row)
        # column split: my slice of the output channels
        mine = parallel.shard_quantized(full_c, parallel.COLUMN, tp, group)
        assert mine["values"].shape == (256 // world, 512)
        y_local = ow.linear_fp32(x, dense(mine))
        gathered = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(gathered, y_local)
        y_full = ow.linear_fp32(x, dense(full_c))
        assert torch.allclose(torch.cat(gathered, -1), y_full, atol=1e-5)
        # row split: my slice of the input channels, partial sums all-reduced
        h = ow.seeded_activation(3, 1024, 4)
        mine = parallel.shard_quantized(full_r, parallel.ROW, tp, group)
        k_local = 1024 // world
        assert mine["values"].shape == (128, k_local) and mine["scale"].shape == (128, k_local // group)
        partial = ow.linear_fp32(h[:, rank * k_local:(rank + 1) * k_local], dense(mine))
        tp.all_reduce(partial)
        assert torch.allclose(partial, ow.linear_fp32(h, dense(full_r)), atol=1e-4)
        # packed runtime buffers of a shard equal the matching slice of the full buffers
        packed_full, scales_full, _ = ow.runtime_buffers(full_r["values"], full_r["scale"], symmetric=not affine,
                                                         zero_point=full_r["zero_point"])
        packed_mine, scales_mine, _ = ow.runtime_buffers(mine["values"], mine["scale"], symmetric=not affine,
                                                         zero_point=mine["zero_point"])
        rows = slice(rank * k_local // 8, (rank + 1) * k_local // 8)
        assert torch.equal(packed_mine, packed_full[rows])
        assert torch.equal(scales_mine, scales_full[rank * k_local // group:(rank + 1) * k_local // group])
    with pytest.raises(ValueError):
        parallel.shard_quantized(full_r, parallel.ROW, parallel.TensorParallel(0, 16), group)
    with pytest.raises(ValueError):
        parallel.TensorParallel(0, 3).check_geometry(4096, 12288, 32, 8, 128)
    parallel.TensorParallel(0, 8).check_geometry(4096, 12288, 32, 8, 128)
    results[rank] = True
    dist.destroy_process_group()


def test_two_rank_sharding_and_all_reduce():
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
        assert dict(results) == {0: True, 1: True}


def test_single_rank_is_identity():
    from linkq2_b200.runtime import parallel
    tp = parallel.TensorParallel()
    data = {"values": torch.zeros(4, 8), "scale": torch.zeros(4, 1), "zero_point": None, "input_scale": None}
    assert parallel.shard_quantized(data, parallel.ROW, tp, 8) is data
    x = torch.ones(2)
    assert tp.all_reduce(x) is x
