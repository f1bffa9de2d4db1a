"""KV4 kernels on the GPU against the golden fixtures and the CPU oracle.

Pool bytes (codes and V scales) and the prefix restore are compared bit for
bit.  Attention outputs use the reference's own tolerance, max |delta| < 2e-3
(``tests/kernels/test_kv4_verify.py:116``, ``test_kv4_materialize.py:73``)."""
import numpy as np
import pytest
import torch

from oracle import kv4 as ok

pytestmark = pytest.mark.gpu

STORE_CASES = ["static_g64", "static_g32_strided", "static_g128", "static_d64"]
ATTN_CASES = ["decode_small", "decode_split", "verify_small", "verify_m16", "verify_neg1", "decode_g32"]
ATOL = 2e-3


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def cuda_pool(kc, vc, word_dtype=torch.int32):
    (kq, ks), (vq, vs) = kc, vc
    kq, vq = kq.cuda(), vq.cuda()
    if word_dtype == torch.uint32:
        kq, vq = kq.view(torch.uint32), vq.view(torch.uint32)
    return (kq, ks.cuda()), (vq, vs.cuda())


def words(x):
    x = x.cpu()
    return x.view(torch.int32) if x.dtype == torch.uint32 else x


@pytest.mark.parametrize("name", STORE_CASES)
@pytest.mark.parametrize("word_dtype", [torch.int32, torch.uint32])
def test_golden_store_and_materialize_bit_exact(golden, name, word_dtype):
    from linkq2_b200.kernels.kv4 import materialize_kv, store_kv_quant
    g = golden("kv4_store")
    tokens, h, d, group, _, strided, slots_total = (int(v) for v in g[f"{name}.meta"])
    k, v = t(g[f"{name}.k"]).cuda(), t(g[f"{name}.v"]).cuda()
    if strided:
        fused = torch.zeros(tokens, h * 3, d, dtype=torch.float16, device="cuda")
        fused[:, h:2 * h], fused[:, 2 * h:] = k, v
        _, k, v = fused.chunk(3, dim=1)
        assert not k.is_contiguous()
    kc, vc = ok.empty_pool(slots_total, h, d, group)
    kc[1].copy_(t(g[f"{name}.ks"]))
    kc, vc = cuda_pool(kc, vc, word_dtype)
    store_kv_quant(k, v, kc, vc, t(g[f"{name}.slots"]).cuda(), v_group=group)
    assert torch.equal(words(kc[0]), t(g[f"{name}.kq"]))
    assert torch.equal(words(vc[0]), t(g[f"{name}.vq"]))
    assert torch.equal(vc[1].cpu(), t(g[f"{name}.vs"]))
    km, vm = materialize_kv(kc, vc, t(g[f"{name}.sel"]).cuda(), v_group=group)
    assert torch.equal(km.cpu(), t(g[f"{name}.km"]))
    assert torch.equal(vm.cpu(), t(g[f"{name}.vm"]))


def test_golden_store_ties_and_saturation(golden):
    from linkq2_b200.kernels.kv4 import store_kv_quant
    g = golden("kv4_store")
    kc = (torch.zeros(4, 1, 8, dtype=torch.int32, device="cuda"), t(g["ties.ks"]).cuda())
    vc = (torch.zeros(4, 1, 8, dtype=torch.int32, device="cuda"),
          torch.zeros(4, 1, 1, dtype=torch.float16, device="cuda"))
    store_kv_quant(t(g["ties.k"]).cuda(), t(g["ties.v"]).cuda(), kc, vc,
                   torch.tensor([2], dtype=torch.int32, device="cuda"), v_group=64)
    assert torch.equal(kc[0].cpu(), t(g["ties.kq"]))
    assert torch.equal(vc[0].cpu(), t(g["ties.vq"]))
    assert torch.equal(vc[1].cpu(), t(g["ties.vs"]))


@pytest.mark.parametrize("group", [32, 64, 128])
def test_store_bit_exact_vs_oracle_at_model_geometry(group):
    """8 KV heads x 128 channels, 300 tokens with outlier channels, shuffled
    slots, a skipped token, int64 slot ids and odd (unaligned) token strides."""
    from linkq2_b200.kernels.kv4 import materialize_kv, store_kv_quant
    tokens, h, d, slots_total = 300, 8, 128, 512
    k, v = ok.seeded_kv(tokens, h, d, seed=group)
    ks = ok.static_k_scale(k)
    g = torch.Generator().manual_seed(1)
    slots = torch.randperm(slots_total, generator=g)[:tokens]
    slots[7] = -1
    ref_k, ref_v = ok.empty_pool(slots_total, h, d, group)
    ref_k[1].copy_(ks)
    ok.store_kv_quant(k, v, ref_k, ref_v, slots, v_group=group)
    for pad in (0, 3):                                   # pad=3 forces the scalar-load path
        wide_k = torch.zeros(tokens, h * d + pad, dtype=torch.float16, device="cuda")
        wide_v = torch.zeros_like(wide_k)
        wide_k[:, :h * d], wide_v[:, :h * d] = k.cuda().flatten(1), v.cuda().flatten(1)
        kk = wide_k[:, :h * d].unflatten(1, (h, d))
        vv = wide_v[:, :h * d].unflatten(1, (h, d))
        kc, vc = ok.empty_pool(slots_total, h, d, group)
        kc[1].copy_(ks)
        kc, vc = cuda_pool(kc, vc, torch.uint32)
        store_kv_quant(kk, vv, kc, vc, slots.cuda(), v_group=group)
        assert torch.equal(words(kc[0]), ref_k[0])
        assert torch.equal(words(vc[0]), ref_v[0])
        assert torch.equal(vc[1].cpu(), ref_v[1])
    sel = torch.tensor([int(slots[0]), int(slots[5]), int(slots[0]), int(slots[299])])
    km, vm = materialize_kv(kc, vc, sel.cuda(), v_group=group)
    rk, rv = ok.materialize_kv(ref_k, ref_v, sel, v_group=group)
    assert torch.equal(km.cpu(), rk) and torch.equal(vm.cpu(), rv)
    empty_k, empty_v = materialize_kv(kc, vc, torch.zeros(0, dtype=torch.int64, device="cuda"), v_group=group)
    assert empty_k.shape == (0, h, d) and empty_v.shape == (0, h, d)


@pytest.mark.parametrize("name", ATTN_CASES)
def test_golden_attention(golden, name):
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    g = golden("kv4_attention")
    bs, m, hq, hkv, d, page, group = (int(v) for v in g[f"{name}.meta"])
    kc = (t(g[f"{name}.kq"]).cuda(), t(g[f"{name}.ks"]).cuda())
    vc = (t(g[f"{name}.vq"]).cuda(), t(g[f"{name}.vs"]).cuda())
    out = paged_attention_decode(t(g[f"{name}.q"]).cuda(), kc, vc, t(g[f"{name}.table"]).cuda(),
                                 t(g[f"{name}.lens"]).cuda(), block_n=page, num_kv_heads=hkv,
                                 v_group=group, verify_m=m)
    ref = t(g[f"{name}.out"]).float()
    assert torch.isfinite(out).all()
    assert (out.float().cpu() - ref).abs().max().item() < ATOL


def build_case(bs, lens, m, hq, hkv, d, page, group, seed, width=None):
    g = torch.Generator().manual_seed(seed)
    blocks = [(l + m + page - 1) // page for l in lens]
    n_blocks = sum(blocks) + 2
    k, v = ok.seeded_kv(n_blocks * page, hkv, d, seed, outlier_channels=4)
    k, v = (k.float() * 0.5).half(), (v.float() * 0.5).half()
    kc, vc = ok.empty_pool(n_blocks * page, hkv, d, group)
    kc[1].copy_(ok.static_k_scale(k))
    ok.store_kv_quant(k, v, kc, vc, torch.arange(n_blocks * page), v_group=group)
    perm = torch.randperm(n_blocks, generator=g).tolist()
    width = width or max(blocks)
    table = torch.full((bs, width), -1, dtype=torch.int32)
    for i, nb in enumerate(blocks):
        ids, perm = perm[:nb], perm[nb:]
        table[i, :nb] = torch.tensor(ids, dtype=torch.int32)
    q = (torch.randn(bs * m, hq, d, generator=g) * 0.5).half()
    return kc, vc, table, torch.tensor(lens, dtype=torch.int32), q


@pytest.mark.parametrize("bs,lens,m,hq,hkv,d,page,group", [
    (1, [2049], 1, 32, 8, 128, 256, 64),        # long context over several splits
    (1, [2049], 16, 32, 8, 128, 256, 64),       # 16-position verify, 64 rows per KV head
    (3, [17, 1000, 256], 1, 16, 8, 128, 256, 64),   # Qwen3-1.7B head geometry, ragged batch
    (2, [300, 31], 16, 16, 8, 128, 256, 64),    # verify with two row tiles
    (2, [1, 500], 1, 4, 4, 64, 32, 32),         # no GQA, single-token context, D = 64
    (4, [0, 5, 0, 40], 1, 8, 2, 128, 16, 128),  # empty sequences yield zeros
    (2, [120, 64], 3, 8, 2, 128, 64, 64),       # odd verify width
    (4, [2100, 700, 2049, 33], 1, 4, 1, 128, 256, 64),   # one KV head per rank: Qwen3-8B at TP = 8
    (2, [2100, 300], 16, 4, 1, 128, 256, 64),   # the same, 16-position verify
    (3, [1500, 2100, 9], 1, 8, 2, 128, 256, 64),         # TP = 4
])
def test_attention_against_oracle(bs, lens, m, hq, hkv, d, page, group):
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    kc, vc, table, ctx, q = build_case(bs, lens, m, hq, hkv, d, page, group, seed=len(lens) + m)
    ref = ok.paged_attention_decode(q, kc, vc, table, ctx, block_n=page, num_kv_heads=hkv,
                                    v_group=group, verify_m=m).float()
    gk, gv = cuda_pool(kc, vc, torch.uint32)
    big = torch.zeros(bs * m, 2 * hq * d, dtype=torch.float16, device="cuda")
    big[:, :hq * d] = q.cuda().flatten(1)
    q_view = big[:, :hq * d].unflatten(1, (hq, d))          # row stride 2*HQ*D, as a fused slice
    out = paged_attention_decode(q_view, gk, gv, table.cuda(), ctx.cuda(), block_n=page,
                                 num_kv_heads=hkv, v_group=group, verify_m=m)
    assert out.shape == (bs * m, hq, d) and out.is_contiguous()
    assert torch.isfinite(out).all()
    assert (out.float().cpu() - ref).abs().max().item() < ATOL
    for i, length in enumerate(lens):
        if length == 0 and m == 1:
            assert not out[i].any()


def test_verify_causality_bit_identical():
    """``tests/kernels/test_kv4_verify.py:120-148`` of the reference: overwriting
    the last draft's slot must leave every earlier row bit-identical."""
    from linkq2_b200.kernels.kv4 import paged_attention_decode, store_kv_quant
    bs, length, m, hq, hkv, d, page = 1, 40, 4, 4, 2, 64, 32
    kc, vc, _, ctx, q = build_case(bs, [length], m, hq, hkv, d, page, 64, seed=3)
    table = torch.arange(kc[0].shape[0] // page, dtype=torch.int32)[None]
    gk, gv = cuda_pool(kc, vc)

    def run():
        return paged_attention_decode(q.cuda(), gk, gv, table.cuda(), ctx.cuda(), block_n=page,
                                      num_kv_heads=hkv, v_group=64, verify_m=m)
    a = run()
    bad = (torch.randn(1, hkv, d) * 10).half().cuda()
    store_kv_quant(bad, bad.flip(-1), gk, gv,
                   torch.tensor([length + m - 2], dtype=torch.int32, device="cuda"), v_group=64)
    b = run()
    assert torch.equal(a[:m - 1], b[:m - 1]), "earlier rows changed"
    assert not torch.equal(a[m - 1], b[m - 1]), "last row did not move"


def test_repeated_block_and_context_swap():
    """``tests/kernels/test_kv4_paged.py:66-115`` of the reference: a block table
    may name one physical block twice, and each sequence uses its own length."""
    from linkq2_b200.kernels.kv4 import paged_attention_decode
    hq, hkv, d, page = 16, 8, 128, 128
    k, v = ok.seeded_kv(8 * page, hkv, d, seed=0)
    kc, vc = ok.empty_pool(8 * page, hkv, d, 64)
    kc[1].copy_(ok.static_k_scale(k))
    ok.store_kv_quant(k, v, kc, vc, torch.arange(8 * page), v_group=64)
    table = torch.tensor([[1, 2, 2], [3, 4, 5]], dtype=torch.int32)
    lens = torch.tensor([200, 300], dtype=torch.int32)
    g = torch.Generator().manual_seed(4)
    q = (torch.randn(2, hq, d, generator=g) * 0.5).half()
    gk, gv = cuda_pool(kc, vc)
    out = paged_attention_decode(q.cuda(), gk, gv, table.cuda(), lens.cuda(), block_n=page, num_kv_heads=hkv)
    ref = ok.paged_attention_decode(q, kc, vc, table, lens, block_n=page, num_kv_heads=hkv)
    assert (out.float().cpu() - ref.float()).abs().max().item() < ATOL
    out2 = paged_attention_decode(q.cuda(), gk, gv, table.cuda(), lens.flip(0).cuda(), block_n=page,
                                  num_kv_heads=hkv)
    assert (out2[0].float() - out[0].float()).abs().max().item() > 1e-3
    again = paged_attention_decode(q.cuda(), gk, gv, table.cuda(), lens.cuda(), block_n=page, num_kv_heads=hkv)
    assert torch.equal(out, again)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_store_takes_wider_inputs_at_full_precision(dtype):
    """The reference's store kernel widens whatever it loads to fp32 (``store.py:31,45``) and its
    own verify test stores fp32 tensors: fp32 and bf16 inputs are quantized from their own
    values, bit for bit as the oracle does from ``k.float()``, also from strided slices."""
    from linkq2_b200.kernels.kv4 import store_kv_quant
    tokens, h, d, slots_total = 70, 2, 128, 128
    g = torch.Generator().manual_seed(12)
    k = (torch.randn(tokens, h, d, generator=g) * 1.7).to(dtype)
    v = (torch.randn(tokens, h, d, generator=g) * 0.9).to(dtype)
    ks = ok.static_k_scale(k.float().half())
    slots = torch.randperm(slots_total, generator=g)[:tokens].int()
    ref_k, ref_v = ok.empty_pool(slots_total, h, d, 64)
    ref_k[1].copy_(ks)
    ok.store_kv_quant(k, v, ref_k, ref_v, slots, v_group=64)
    for pad in (0, 3):
        wide = torch.zeros(tokens, 2 * h * d + pad, dtype=dtype, device="cuda")
        wide[:, :h * d], wide[:, h * d:2 * h * d] = k.cuda().flatten(1), v.cuda().flatten(1)
        kc, vc = ok.empty_pool(slots_total, h, d, 64)
        kc[1].copy_(ks)
        kc, vc = cuda_pool(kc, vc, torch.uint32)
        store_kv_quant(wide[:, :h * d].unflatten(1, (h, d)), wide[:, h * d:2 * h * d].unflatten(1, (h, d)),
                       kc, vc, slots.cuda(), v_group=64)
        assert torch.equal(words(kc[0]), ref_k[0])
        assert torch.equal(words(vc[0]), ref_v[0])
        assert torch.equal(vc[1].cpu(), ref_v[1])


@pytest.mark.parametrize("hq,hkv,d,page,group,rows,prefixes", [
    (32, 8, 128, 256, 64, 16, [700, 2100, 0, 33]),          # verify kernel, several splits, an empty prefix
    (16, 8, 128, 128, 64, 16, [257, 1000]),                 # two heads per group: 32 rows per KV head
    (4, 2, 64, 128, 32, 16, [300, 90]),                     # D = 64: the generic kernel
    (8, 1, 128, 128, 128, 8, [513, 40, 1300]),              # eight heads per group: blocks of 8 rows
])
def test_prefix_attention_against_oracle(hq, hkv, d, page, group, rows, prefixes):
    """The pool half of chunked prefill: out and log-sum-exp against the oracle on dequantised slots,
    and merging it with an fp32 attention over extra keys equals attention over both."""
    from linkq2_b200.kernels.kv4.ops import paged_attention_prefix
    g = torch.Generator().manual_seed(hq + d)
    blocks = [(n + page - 1) // page for n in prefixes]
    n_blocks = sum(blocks) + 2
    k, v = ok.seeded_kv(n_blocks * page, hkv, d, seed=d + rows, outlier_channels=2)
    kc, vc = ok.empty_pool(n_blocks * page, hkv, d, group)
    kc[1].copy_(ok.static_k_scale(k))
    ok.store_kv_quant(k, v, kc, vc, torch.arange(n_blocks * page), v_group=group)
    perm = torch.randperm(n_blocks, generator=g).tolist()
    table = torch.full((len(prefixes), max(max(blocks), 1)), -1, dtype=torch.int32)
    for i, nb in enumerate(blocks):
        table[i, :nb] = torch.tensor(perm[:nb], dtype=torch.int32)
        perm = perm[nb:]
    lens = torch.tensor(prefixes, dtype=torch.int32)
    q = (torch.randn(len(prefixes) * rows, hq, d, generator=g) * 0.7).half()
    gk, gv = cuda_pool(kc, vc)
    out, lse = paged_attention_prefix(q.cuda(), gk, gv, table.cuda(), lens.cuda(), block_n=page, num_kv_heads=hkv,
                                      v_group=group, rows=rows)
    ref, ref_lse = ok.paged_attention_prefix(q, kc, vc, table, lens, block_n=page, num_kv_heads=hkv,
                                             v_group=group, rows=rows)
    # fp16 outputs up to ~15 with the x10 channels: 2e-3 plus the output's own rounding
    assert bool(((out.float().cpu() - ref).abs() <= ATOL + ref.abs() * 2.0 ** -11).all())
    live = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), live)
    assert (lse.cpu()[live] - ref_lse[live]).abs().max().item() < 2e-3
    assert (out.float().cpu()[~live] == 0).all()


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (16, 8, 128), (4, 2, 64), (8, 1, 128)])
def test_chunk_attention_merges_own_rows_with_prefix_part(hq, hkv, d):
    """A step of four sequences - 64 rows with a prefix part, 5 and 40 rows without, 7 rows that
    the caller handles elsewhere - read through strided views of one fused buffer."""
    from linkq2_b200.kernels.kv4.ops import chunk_attention
    g = torch.Generator().manual_seed(hq * d)
    counts = [64, 5, 40, 7]
    t = sum(counts)
    fused = (torch.randn(t, hq + 2 * hkv, d, generator=g) * 0.8).half()
    fused[:, hq:hq + hkv, 3] *= 6                                   # an outlier channel in K
    q, k, v = fused[:, :hq], fused[:, hq:hq + hkv], fused[:, hq + hkv:]
    first, where, at = [], [], 0
    for i, n in enumerate(counts):
        first += [at] * n
        where += list(range(n)) if i == 0 else [-1 if i < 3 else -2] * n
        at += n
    first, where = torch.tensor(first, dtype=torch.int32), torch.tensor(where, dtype=torch.int32)
    pre = (torch.randn(64, hq, d, generator=g) * 0.5).half()
    pre_lse = torch.randn(64, hq, generator=g) * 3 + 2
    pre_lse[5] = float("-inf")                                       # an empty prefix part counts for nothing
    pre_lse[9] = 40.0                                                # a dominant one takes the row over
    gf = fused.cuda()
    out = torch.full((t, hq, d), 7.0, dtype=torch.float16, device="cuda")
    chunk_attention(gf[:, :hq], gf[:, hq:hq + hkv], gf[:, hq + hkv:], first.cuda(), where.cuda(), pre.cuda(),
                    pre_lse.cuda(), out)
    ref = ok.chunk_attention(q, k, v, first, where, pre, pre_lse)
    got = out.float().cpu()
    done = where >= -1
    assert bool(((got[done] - ref[done]).abs() <= ATOL + ref[done].abs() * 2.0 ** -11).all())
    assert bool((got[~done] == 7.0).all())                           # untouched rows
    assert (got[9] - pre[9].float()).abs().max().item() < 1e-3
