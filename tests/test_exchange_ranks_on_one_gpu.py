"""The pushed tensor-parallel exchange for 2, 4 and 8 ranks, all of them emulated on one GPU.

Every emulated rank has an exchange buffer of its own on the same device and the table of all
of them.  A step first runs the row-split projection of every rank, whose epilogue stores the
partial sums into all the buffers (``lq2_w4a16_linear_push``), and only then the gathering
residual RMSNorm of every rank (``lq2_rmsnorm_allreduce_pushed``): by the time a gather is
launched, everything it looks for has been written by kernels that completed before it in the
stream, so no launch ever waits for another one.  This covers the eight-rank instantiation of
the gather (peers requested in groups of four) and the projection's stores to seven peers
without needing eight GPUs; results must have the bits of the rank-ordered fp32 sum and be the
same on every rank, for consecutive steps (which alternate the two halves of the buffers)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _local_exchanges(world, max_bytes):
    from linkq2_b200 import _lib
    from linkq2_b200.runtime.parallel import PeerExchange
    lib = _lib.lib
    size = lib.lq2_allreduce_buffer_bytes(world, max_bytes)
    assert size > 0
    bufs = []
    for _ in range(world):
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        assert lib.lq2_allreduce_buffer_create(size, ctypes.byref(ptr), handle) == 0
        bufs.append(ptr.value)
    table = (ctypes.c_void_p * world)(*bufs)
    exchanges = [PeerExchange(r, world, max_bytes, bufs[r], table, [bufs[r]] + [None] * (world - 1))
                 for r in range(world)]
    return lib, bufs, exchanges


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("rows,k,hidden", [(32, 256, 4096), (16, 512, 2048), (64, 256, 8192), (9, 384, 1024)])
def test_pushed_exchange_of_emulated_ranks(world, rows, k, hidden):
    from linkq2_b200.kernels.fused import rmsnorm, rmsnorm_allreduce
    from linkq2_b200.runtime.backends import make_quant_linear
    torch.cuda.set_device(0)
    max_bytes = 1 << 20
    lib, bufs, exchanges = _local_exchanges(world, max_bytes)
    try:
        before = exchanges[0].timeouts()
        g = torch.Generator().manual_seed(7 * world + rows)
        layers = []
        for r in range(world):
            vals = (torch.randint(0, 16, (hidden, k), generator=g, dtype=torch.uint8).to(torch.int16) - 8).to(torch.int8)
            scale = (torch.rand(hidden, k // 128, generator=g) * 0.01 + 0.001).half()
            layers.append(make_quant_linear("b200", vals, scale, group_size=128, symmetric=True, device="cuda",
                                            dtype=torch.float16))
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).half().cuda()
        for step in range(3):
            xs = [(torch.randn(rows, k, generator=g) * (1 + r)).half().cuda() for r in range(world)]
            res = torch.randn(rows, hidden, generator=g).half().cuda()
            parts = [layers[r](xs[r]) for r in range(world)]
            acc = torch.zeros(rows, hidden, dtype=torch.float32, device="cuda")
            for part in parts:                              # rank order, fp32, one rounding at the end
                acc += part.float()
            want_out, want_res = rmsnorm(acc.half(), w, 1e-6, res)
            pushed = [layers[r].forward_push(xs[r], exchanges[r]) for r in range(world)]
            got = [rmsnorm_allreduce(pushed[r], w, 1e-6, res, exchanges[r], pushed=True) for r in range(world)]
            torch.cuda.synchronize()
            for r in range(world):
                assert torch.equal(pushed[r], parts[r]), (step, r)
                assert torch.equal(got[r][1], want_res), (step, r)
                assert torch.equal(got[r][0], want_out), (step, r)
        assert exchanges[0].timeouts() == before
    finally:
        for b in bufs:
            lib.lq2_allreduce_buffer_close(b, 1)


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("world", [4, 8])
def test_sending_exchange_reaches_the_rank_launched_last(world, fused):
    """The sending variants (``lq2_rmsnorm_allreduce`` and the plain ``lq2_allreduce_fp16``: every
    rank stores its own rows into all buffers, then gathers) with the emulated ranks launched
    one after the other.  Only the rank
    launched last can find all its peers' rows, so only its result is checked; the earlier ones
    run against a budget of a few thousand polls, give up and are counted - the bounded wait
    at work, nothing hangs.  The last rank rotates, so every rank is the receiver once."""
    from linkq2_b200.kernels.fused import rmsnorm, rmsnorm_allreduce
    torch.cuda.set_device(0)
    max_bytes = 1 << 20
    lib, bufs, exchanges = _local_exchanges(world, max_bytes)
    previous = exchanges[0].set_poll_limit(2000)
    try:
        g = torch.Generator().manual_seed(world)
        rows, hidden = 32, 4096
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).half().cuda()
        for last in range(world):
            xs = [(torch.randn(rows, hidden, generator=g) * (1 + r)).half().cuda() for r in range(world)]
            res = torch.randn(rows, hidden, generator=g).half().cuda()
            acc = torch.zeros(rows, hidden, dtype=torch.float32, device="cuda")
            for x in xs:
                acc += x.float()
            want_out, want_res = rmsnorm(acc.half(), w, 1e-6, res)
            order = [r for r in range(world) if r != last] + [last]
            before = exchanges[0].timeouts()
            def run(r):
                if fused:
                    return rmsnorm_allreduce(xs[r], w, 1e-6, res, exchanges[r])
                return exchanges[r].all_reduce(xs[r].clone())
            for r in order[:-1]:
                run(r)
            gave_up = exchanges[0].timeouts()
            assert gave_up > before
            got = run(last)
            torch.cuda.synchronize()
            assert exchanges[0].timeouts() == gave_up, "the rank launched last found everything it waited for"
            if fused:
                assert torch.equal(got[1], want_res) and torch.equal(got[0], want_out), last
            else:
                assert torch.equal(got, acc.half()), last
    finally:
        exchanges[0].set_poll_limit(previous)
        for b in bufs:
            lib.lq2_allreduce_buffer_close(b, 1)
