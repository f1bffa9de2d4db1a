"""Fused elementwise kernels against the reference's eager torch expressions
evaluated on CPU in fp32 (floating-point kernels: tolerance one to two fp16
units in the last place), and the cache bytes of the fused pre-attention kernel
against the KV4 store oracle applied to that kernel's own fp16 keys (bit-exact)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import kv4 as ok

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-3, 2e-3        # fp16 has a 2^-11 relative step; inputs are O(1)


def ref_rmsnorm(x, w, eps, residual=None):
    """qslab/runtime/model/primitives.py:15-30."""
    if residual is None:
        x32 = x.float()
        return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).half() * w, None
    x32 = x.float() + residual.float()
    res = x32.half()
    return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).half() * w, res


@pytest.mark.parametrize("rows,hidden", [(1, 4096), (32, 4096), (5, 2048), (3, 128), (64, 8192), (2, 1536)])
def test_rmsnorm_matches_reference_expression(rows, hidden):
    from linkq2_b200.kernels.fused import rmsnorm
    g = torch.Generator().manual_seed(hidden + rows)
    x = (torch.randn(rows, hidden, generator=g) * 2).half()
    res = torch.randn(rows, hidden, generator=g).half()
    w = (1 + 0.2 * torch.randn(hidden, generator=g)).half()
    y = rmsnorm(x.cuda(), w.cuda(), 1e-6).cpu()
    torch.testing.assert_close(y.float(), ref_rmsnorm(x, w, 1e-6)[0].float(), rtol=RTOL, atol=ATOL)
    y2, r2 = rmsnorm(x.cuda(), w.cuda(), 1e-6, res.cuda())
    ey, er = ref_rmsnorm(x, w, 1e-6, res)
    assert torch.equal(r2.cpu(), er)                       # fp16(x + residual) is exact arithmetic
    torch.testing.assert_close(y2.cpu().float(), ey.float(), rtol=RTOL, atol=ATOL)
    wide = torch.zeros(rows, hidden * 2, dtype=torch.float16, device="cuda")
    wide[:, :hidden] = x.cuda()
    assert torch.equal(rmsnorm(wide[:, :hidden], w.cuda(), 1e-6).cpu(), y)   # row-strided input


def test_silu_mul_matches_reference_expression():
    from linkq2_b200.kernels.fused import silu_mul
    g = torch.Generator().manual_seed(1)
    gate = (torch.randn(7, 12288, generator=g) * 3).half()
    up = torch.randn(7, 12288, generator=g).half()
    expected = F.silu(gate.float()).half() * up
    got = silu_mul(gate.cuda(), up.cuda()).cpu()
    torch.testing.assert_close(got.float(), expected.float(), rtol=RTOL, atol=ATOL)
    both = torch.cat([gate, up], -1).cuda()                # slices of a fused gate_up buffer
    assert torch.equal(silu_mul(both[:, :12288], both[:, 12288:]).cpu(), got)


def ref_pre_attention(q, k, qw, kw, cos_sin, positions, eps, lam):
    """qwen3.py:49-51, rotary.py:12-16,103-108, attention.py:72-77 on CPU."""
    def norm(x, w):
        x32 = x.float()
        return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).half() * w

    def rope(x):
        cos, sin = cos_sin[positions].chunk(2, dim=-1)
        x1, x2 = torch.chunk(x.float(), 2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).half()
    q, k = rope(norm(q, qw)), rope(norm(k, kw))
    if lam is not None:
        rep = q.shape[1] // k.shape[1]
        q = q * lam.repeat_interleave(rep, 0)
        k = k / lam
    return q, k


@pytest.mark.parametrize("d,hq,hkv,group", [(128, 32, 8, 64), (128, 4, 1, 32), (128, 16, 8, 128),
                                            (64, 2, 1, 64), (64, 4, 2, 32)])
@pytest.mark.parametrize("with_lambda", [False, True])
def test_pre_attention_numerics_and_cache_bytes(d, hq, hkv, group, with_lambda):
    from linkq2_b200.kernels.fused import pre_attention
    from linkq2_b200.runtime.model.rotary import RotaryEmbedding
    tokens, slots_total = 37, 64
    g = torch.Generator().manual_seed(d + hq + group)
    fused = torch.randn(tokens, (hq + 2 * hkv) * d, generator=g).half()
    q, k, v = fused.split([hq * d, hkv * d, hkv * d], dim=-1)
    q, k, v = q.unflatten(1, (hq, d)), k.unflatten(1, (hkv, d)), v.unflatten(1, (hkv, d))
    qw = (1 + 0.1 * torch.randn(d, generator=g)).half()
    kw = (1 + 0.1 * torch.randn(d, generator=g)).half()
    rope = RotaryEmbedding(d, 512, 1e6)
    positions = torch.randint(0, 512, (tokens,), generator=g)
    lam = (0.5 + torch.rand(hkv, d, generator=g)).half() if with_lambda else None
    slots = torch.randperm(slots_total, generator=g)[:tokens].int()
    slots[3] = -1
    kc, vc = ok.empty_pool(slots_total, hkv, d, group)
    kc[1].copy_((torch.rand(hkv, d, generator=g) * 0.3 + 0.1).half())
    gq, gk, gv = (t.unflatten(1, (-1, d)) for t in fused.cuda().split([hq * d, hkv * d, hkv * d], dim=-1))
    assert not gk.is_contiguous()
    gkc = (kc[0].clone().cuda(), kc[1].cuda())
    gvc = (vc[0].clone().cuda(), vc[1].clone().cuda())
    lam_q = None if lam is None else lam.repeat_interleave(hq // hkv, 0).contiguous().cuda()
    q_out, k_out = pre_attention(gq, gk, gv, qw.cuda(), kw.cuda(), rope.cos_sin_cache.cuda(), positions.cuda(), 1e-6,
                                 lam_q=lam_q, lam_k=None if lam is None else lam.cuda(), k_cache=gkc, v_cache=gvc,
                                 slot_mapping=slots.cuda(), v_group=group, want_k=True)
    eq, ek = ref_pre_attention(q, k, qw, kw, rope.cos_sin_cache, positions, 1e-6, lam)
    torch.testing.assert_close(q_out.cpu().float(), eq.float(), rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(k_out.cpu().float(), ek.float(), rtol=RTOL, atol=ATOL)
    # the pool holds exactly the KV4 encoding of the kernel's own fp16 keys and of v
    ok.store_kv_quant(k_out.cpu(), v.contiguous(), kc, vc, slots, v_group=group)
    assert torch.equal(gkc[0].cpu(), kc[0]) and torch.equal(gvc[0].cpu(), vc[0])
    assert torch.equal(gvc[1].cpu(), vc[1])
    # without a slot mapping nothing is stored and k_out can be skipped
    q2, none = pre_attention(gq, gk, gv, qw.cuda(), kw.cuda(), rope.cos_sin_cache.cuda(), positions.cuda(), 1e-6,
                             lam_q=lam_q, lam_k=None if lam is None else lam.cuda())
    assert none is None and torch.equal(q2, q_out)
