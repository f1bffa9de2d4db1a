"""The allocation-free KV4 attention entry point, called through the C ABI.

``lq2_kv4_attention_static`` keeps its split partials in an array built into the
library, for hosts that cannot hand the library a workspace (they own no
allocator the plugin can reach, or must not allocate where they call it).  It
runs the same kernel as ``lq2_kv4_attention``, so the two must agree; the check
uses the 2e-3 tolerance of the other attention tests and runs the call twice in
a row, because the second call finds the array as the first one left it.
This file sorts last so that a run stopping at the first failure has already
run every other test.
"""
import pytest
import torch

from oracle import kv4 as ok

pytestmark = pytest.mark.gpu

ATOL = 2e-3


def _case(bs, lens, m, hq, hkv, d, page, seed):
    g = torch.Generator().manual_seed(seed)
    blocks = [(l + m + page - 1) // page for l in lens]
    n_blocks = sum(blocks) + 1
    k, v = ok.seeded_kv(n_blocks * page, hkv, d, seed)
    kc, vc = ok.empty_pool(n_blocks * page, hkv, d, 64)
    kc[1].copy_(ok.static_k_scale(k))
    ok.store_kv_quant(k, v, kc, vc, torch.arange(n_blocks * page), v_group=64)
    perm = torch.randperm(n_blocks, generator=g).tolist()
    table = torch.full((bs, max(blocks)), -1, dtype=torch.int32)
    for i, nb in enumerate(blocks):
        table[i, :nb] = torch.tensor(perm[:nb], dtype=torch.int32)
        perm = perm[nb:]
    q = (torch.randn(bs * m, hq, d, generator=g) * 0.5).half()
    return kc, vc, table, torch.tensor(lens, dtype=torch.int32), q


def _static_call(q, kc, vc, table, lens, m, hkv, page, out=None):
    """Raw ctypes call: pointers, sizes and the current stream; no workspace."""
    from linkq2_b200 import _lib
    rows, hq, d = q.shape
    out = torch.empty_like(q) if out is None else out
    status = _lib.lib.lq2_kv4_attention_static(
        q.data_ptr(), q.stride(0), kc[0].data_ptr(), kc[1].data_ptr(), vc[0].data_ptr(), vc[1].data_ptr(),
        table.data_ptr(), lens.data_ptr(), out.data_ptr(), rows // m, m, hq, hkv, d, page, table.shape[1],
        64, kc[0].shape[0], torch.cuda.current_stream().cuda_stream)
    return status, out


@pytest.mark.parametrize("bs,lens,m", [(2, [1500, 700], 1), (1, [1200], 16)])
def test_static_scratch_matches_workspace_entry_twice(bs, lens, m):
    from linkq2_b200 import _lib
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    hq, hkv, d, page = 32, 8, 128, 256
    kc, vc, table, ctx, q = _case(bs, lens, m, hq, hkv, d, page, seed=bs + m)
    assert _lib.lib.lq2_kv4_attention_splits(bs, m, hq, hkv, d, page, table.shape[1]) > 1   # scratch is used
    gk = (kc[0].cuda(), kc[1].cuda())
    gv = (vc[0].cuda(), vc[1].cuda())
    table, ctx, q = table.cuda(), ctx.cuda(), q.cuda()
    expected = paged_attention_decode(q, gk, gv, table, ctx, block_n=page, num_kv_heads=hkv, verify_m=m)
    before = torch.cuda.memory_allocated()
    for call in range(2):
        out = torch.empty_like(q)                            # the caller's output, allocated before the call
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]           # device-wide free bytes (cudaMemGetInfo)
        status, out = _static_call(q, gk, gv, table, ctx, m, hkv, page, out)
        assert status == _lib.OK
        torch.cuda.synchronize()
        if call == 1:                                        # the first call on a device may load the module
            assert torch.cuda.mem_get_info()[0] >= free_before, "the call took device memory"
        assert (out.float() - expected.float()).abs().max().item() < ATOL
    del out
    assert torch.cuda.memory_allocated() == before           # nothing was taken from torch's pool either
    ref = ok.paged_attention_decode(q.cpu(), kc, vc, table.cpu(), ctx.cpu(), block_n=page, num_kv_heads=hkv,
                                    verify_m=m)
    assert (expected.float().cpu() - ref.float()).abs().max().item() < ATOL


def test_static_scratch_rejects_oversized_problem():
    from linkq2_b200 import _lib
    limit = _lib.lib.lq2_kv4_attention_static_max_bytes()
    assert limit == 16 << 20
    bs, m, hq, hkv, d, page, blocks = 64, 16, 32, 8, 128, 256, 128
    assert _lib.lib.lq2_kv4_attention_workspace_bytes(bs, m, hq, hkv, d, page, blocks) > limit
    fake = 1 << 20       # never dereferenced: the call is refused before any launch
    status = _lib.lib.lq2_kv4_attention_static(fake, hq * d, fake, fake, fake, fake, fake, fake, fake, bs, m, hq,
                                               hkv, d, page, blocks, 64, blocks * page * bs, None)
    assert status == _lib.ERR_LIMIT
    assert b"16 MiB" in _lib.lib.lq2_status_string(status)
