"""A bounded wait of the tensor-parallel exchange kernels, made to run out on one GPU.

``world = 2`` with both table entries local allocations: the "peer" buffer is a second buffer
on the same GPU that nothing ever writes into this rank's slots, so every thread of the
kernel waits for data that cannot arrive.  With a limit of a few thousand polls the kernel
must return promptly, the abandoned waits must be counted, the status must reach the host
wrapper, and the context must stay usable.  Nothing faults and nothing spins on another
launch; the wait simply ends."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _two_local_buffers(lib, max_bytes):
    size = lib.lq2_allreduce_buffer_bytes(2, max_bytes)
    assert size > 0
    bufs = []
    for _ in range(2):
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        assert lib.lq2_allreduce_buffer_create(size, ctypes.byref(ptr), handle) == 0
        bufs.append(ptr.value)
    return bufs


@pytest.mark.parametrize("fused", [True, False])
def test_exchange_wait_runs_out_and_is_reported(fused):
    from linkq2_b200 import _lib
    from linkq2_b200.runtime.parallel import PeerExchange
    lib = _lib.lib
    torch.cuda.set_device(0)
    max_bytes = 1 << 20
    bufs = _two_local_buffers(lib, max_bytes)
    table = (ctypes.c_void_p * 2)(*bufs)
    exchange = PeerExchange(0, 2, max_bytes, bufs[0], table, [bufs[0], None])
    previous = exchange.set_poll_limit(5000)
    try:
        before = exchange.timeouts()
        rows, hidden = 4, 8192                              # four chunks per thread in the fused kernel
        x = torch.randn(rows, hidden, device="cuda", dtype=torch.float16)
        stream = torch.cuda.current_stream().cuda_stream
        torch.cuda.synchronize()
        t0 = time.time()
        if fused:
            res = torch.zeros_like(x)
            w = torch.ones(hidden, device="cuda", dtype=torch.float16)
            out, res_out = torch.empty_like(x), torch.empty_like(x)
            status = lib.lq2_rmsnorm_allreduce(x.data_ptr(), hidden, res.data_ptr(), w.data_ptr(), out.data_ptr(),
                                               res_out.data_ptr(), rows, hidden, 1e-6, table, 0, 2, max_bytes, stream)
        else:
            status = lib.lq2_allreduce_fp16(x.data_ptr(), x.data_ptr(), x.numel(), table, 0, 2, max_bytes, stream)
        assert status == 0
        torch.cuda.synchronize()
        elapsed = time.time() - t0
        assert elapsed < 5.0, f"the kernel took {elapsed:.1f} s to give up"
        after = exchange.timeouts()
        assert after > before
        with pytest.raises(RuntimeError, match="abandoned waits"):
            exchange.check()
        # the context is still usable
        y = torch.ones(1024, device="cuda") * 2
        assert float(y.sum()) == 2048.0
    finally:
        exchange.set_poll_limit(previous)
        for b in bufs:
            lib.lq2_allreduce_buffer_close(b, 1)
