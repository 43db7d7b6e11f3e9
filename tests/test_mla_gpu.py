"""Sparse-MLA kernels (RoPE, cache writes, fp8 indexer on tcgen05, top-k,
latent attention on tcgen05) vs the fp32 references."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.oracle import mla as ref

pytestmark = pytest.mark.gpu


def _rel(y, r):
    return ((y.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("interleaved", [False, True])
def test_rope(interleaved):
    torch.manual_seed(0)
    cs = ref.rope_cos_sin(4096, 64).cuda()
    x = torch.randn(9, 5, 192, dtype=torch.bfloat16, device="cuda")
    pos = torch.randint(0, 4096, (9,), dtype=torch.int32, device="cuda")
    r = ref.rope(x.cpu(), pos.cpu(), cs.cpu(), 128, 64, interleaved)
    _ext.ops().rope(x, pos, cs, 128, 64, interleaved)
    assert _rel(x.cpu(), r) < 1e-2


def test_latent_cache_write():
    torch.manual_seed(0)
    cs = ref.rope_cos_sin(1024, 64).cuda()
    T = 13
    kv = torch.randn(T, 576, dtype=torch.bfloat16, device="cuda")
    w = torch.randn(512, dtype=torch.bfloat16, device="cuda")
    pos = torch.randint(0, 1024, (T,), dtype=torch.int32, device="cuda")
    slots = torch.randperm(64, device="cuda")[:T].long()
    cache = torch.zeros(64, 576, dtype=torch.bfloat16, device="cuda")
    _ext.ops().mla_latent_cache_write(kv, w, 1e-6, pos, cs, False, slots, cache)
    r = ref.latent_row(kv.cpu(), w.cpu(), 1e-6, pos.cpu(), cs.cpu(), False)
    assert _rel(cache[slots].cpu(), r) < 1e-2


def _make_index(T_ctx, nseq=2, bs=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    cs = ref.rope_cos_sin(8192, 64)
    nblk = (T_ctx + bs - 1) // bs
    bt = torch.randperm(nseq * nblk + 5, generator=g)[: nseq * nblk].view(nseq, nblk).int()
    k_raw = torch.randn(nseq, T_ctx, 128, generator=g).to(torch.bfloat16)
    return cs, bt, k_raw


def test_indexer_and_topk():
    torch.manual_seed(0)
    nseq, ctx, bs = 2, 700, 64
    cs, bt, k_raw = _make_index(ctx, nseq, bs)
    ops = _ext.ops()
    nslots = (bt.max().item() + 1) * bs
    kc = torch.zeros(nslots, 128, dtype=torch.uint8, device="cuda")
    ks = torch.zeros(nslots, dtype=torch.float32, device="cuda")
    ln_w = (1 + 0.1 * torch.randn(128)).to(torch.bfloat16)
    for s in range(nseq):
        pos = torch.arange(ctx, dtype=torch.int32)
        slots = (bt[s][pos // bs].long() * bs + pos % bs)
        ops.mla_index_k_write(k_raw[s].cuda(), ln_w.cuda(), None, 1e-6, pos.cuda(), cs.cuda(), False, slots.cuda(), kc,
                              ks)
    # keys: kernel fp8 vs reference (fp8 tolerance)
    pos = torch.arange(ctx, dtype=torch.int32)
    kref = ref.index_k(k_raw[0], ln_w, None, 1e-6, pos, cs, False)
    slots0 = (bt[0][pos // bs].long() * bs + pos % bs)
    kdeq = kc[slots0.cuda()].view(torch.float8_e4m3fn).float().cpu() * ks[slots0.cuda()].cpu()[:, None]
    assert _rel(kdeq, kref) < 0.06
    # queries: 3 tokens of seq 0 and 2 of seq 1 at various context lengths
    T = 5
    token_seq = torch.tensor([0, 0, 1, 0, 1], dtype=torch.int32)
    ctx_lens = torch.tensor([1, 65, 300, 700, 128], dtype=torch.int32)
    qraw = torch.randn(T, 64, 128).to(torch.bfloat16)
    w = torch.randn(T, 64).to(torch.bfloat16)
    q8 = torch.empty(T, 64, 128, dtype=torch.uint8, device="cuda")
    wo = torch.empty(T, 64, dtype=torch.float32, device="cuda")
    qpos = (ctx_lens - 1).cuda()
    ops.mla_index_q_prep(qraw.cuda(), qpos, cs.cuda(), False, w.cuda(), 0.125, q8, wo)
    scores = torch.full((T, 768), float("nan"), dtype=torch.float32, device="cuda")
    st = _ext.status_word(torch.device("cuda"))
    ops.mla_indexer_scores(q8, wo, kc, ks, ctx_lens.cuda(), token_seq.cuda(), bt.cuda(), 768, scores, st)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    qdeq = q8.view(torch.float8_e4m3fn).float().cpu()
    for t in range(T):
        s = int(token_seq[t])
        c = int(ctx_lens[t])
        p = torch.arange(c)
        sl = (bt[s][p // bs].long() * bs + p % bs).cuda()
        keys = kc[sl].view(torch.float8_e4m3fn).float().cpu() * ks[sl].cpu()[:, None]
        r = ref.indexer_scores(qdeq[t], wo[t].cpu(), keys)
        assert _rel(scores[t, :c].cpu(), r) < 1e-4, t
    # top-k on these scores (k = 256), with forced ties
    scores[3, 10:20] = scores[3, 400]
    out = torch.empty(T, 256, dtype=torch.int32, device="cuda")
    cnt = torch.empty(T, dtype=torch.int32, device="cuda")
    ops.mla_topk(scores, ctx_lens.cuda(), 256, token_seq.cuda(), bt.cuda(), bs, out, cnt)
    for t in range(T):
        s, c = int(token_seq[t]), int(ctx_lens[t])
        p = ref.topk_positions(scores[t].cpu(), c, 256)
        exp = (bt[s][p // bs].long() * bs + p % bs).int()
        assert int(cnt[t]) == len(p)
        assert torch.equal(out[t, : len(p)].cpu(), exp), t
        assert (out[t, len(p):] == -1).all()


@pytest.mark.parametrize("nh,count,splits,qscale", [(128, 2048, 1, 0.3), (32, 2048, 1, 0.3), (16, 100, 1, 0.3),
                                                    (64, 1000, 3, 0.3), (128, 64, 2, 0.3), (8, 257, 1, 0.3),
                                                    (128, 2048, 8, 0.3), (32, 1500, 1, 3.0), (160, 700, 2, 0.3),
                                                    (4, 300, 1, 0.3), (4, 2048, 2, 0.3)])
def test_sparse_attention(nh, count, splits, qscale):
    """qscale 3.0 gives logit ranges that force rescaling across the 256-position blocks;
    nh 160 spans two head groups; count 257 ends one position into a second block."""
    torch.manual_seed(nh + count)
    T, topk, nslots = 3, 2048, 5000
    cache = torch.randn(nslots, 576, dtype=torch.bfloat16, device="cuda")
    q = (torch.randn(T, nh, 576, device="cuda") * qscale).to(torch.bfloat16)
    idx = torch.full((T, topk), -1, dtype=torch.int32, device="cuda")
    counts = torch.tensor([count, max(1, count // 2), count], dtype=torch.int32, device="cuda")
    for t in range(T):
        c = int(counts[t])
        idx[t, :c] = torch.randperm(nslots, device="cuda")[:c].sort().values.int()
    out = torch.empty(T, nh, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(T, nh, dtype=torch.float32, device="cuda")
    scale = 192 ** -0.5
    _ext.ops().mla_sparse_attention(q, cache, idx, counts, scale, splits, out, lse, _ext.status_word(q.device))
    torch.cuda.synchronize()
    _ext.check_status(q.device)
    for t in range(T):
        c = int(counts[t])
        rows = cache[idx[t, :c].long()].cpu()
        o_r, lse_r = ref.sparse_attention(q[t].cpu(), rows, scale)
        assert _rel(out[t].cpu(), o_r) < 2e-2, (t, _rel(out[t].cpu(), o_r))
        assert (lse[t].cpu() - lse_r).abs().max() < 2e-2


@pytest.mark.parametrize("H", [1, 2, 3])
@pytest.mark.parametrize("n", [8, 64, 256])
def test_batched_head_gemms(H, n):
    """The MLA absorb and up-projection GEMMs on per-head views (`ops.bmm`: [H, n, K] slices of [n, H, D]
    tensors, outputs written into slices of wider rows) against fp32 per-head matmuls; one head (a
    rank's share of a small model) takes the 2-D path."""
    from vllm_cmp170hx_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(H * 1000 + n)
    q = torch.randn(n, H, 192, device="cuda", generator=g).bfloat16()
    w_uk_t = (torch.randn(H + 1, 512, 128, device="cuda", generator=g) * 0.1).bfloat16()
    qf = torch.zeros(n, H, 576, dtype=torch.bfloat16, device="cuda")
    ops.bmm(q[:, :, :128].transpose(0, 1), w_uk_t[1:1 + H], out=qf[:, :, :512].transpose(0, 1))
    ref = torch.einsum("nhk,hjk->nhj", q[:, :, :128].float(), w_uk_t[1:1 + H].float())
    assert ((qf[:, :, :512].float() - ref).norm() / ref.norm()).item() < 1e-2
    assert qf[:, :, 512:].abs().max().item() == 0  # the rope columns of the rows are untouched
    o_lat = torch.randn(n, H, 512, device="cuda", generator=g).bfloat16()
    w_uv = (torch.randn(H, 128, 512, device="cuda", generator=g) * 0.05).bfloat16()
    o = torch.empty(n, H * 128, dtype=torch.bfloat16, device="cuda")
    ops.bmm(o_lat.transpose(0, 1), w_uv, out=o.view(n, H, 128).transpose(0, 1))
    ref2 = torch.einsum("nhk,hjk->nhj", o_lat.float(), w_uv.float()).reshape(n, H * 128)
    assert ((o.float() - ref2).norm() / ref2.norm()).item() < 1e-2
