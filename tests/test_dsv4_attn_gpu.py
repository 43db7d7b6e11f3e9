"""DeepSeek-V4.1 attention on the GPU: the 512-wide block-sparse attention kernel with per-head
sinks (csrc/mla_attn.cu, D = 512) against the fp32 oracle, unsplit and split over positions (the
sink then enters in the merge), and the cached core on CUDA against the same core on the host."""

import pytest
import torch

from vllm_cmp170hx_b200.oracle import dsv4_attn as ref
from vllm_cmp170hx_b200.ops.dsv4_attn import DSv4AttnCore, DSv4AttnSpec, attend

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,h,splits", [(5, 64, 1), (3, 64, 3), (9, 8, 1), (2, 128, 2), (4, 16, 4)])
def test_sink_attention_matches_oracle(T, h, splits):
    g = torch.Generator().manual_seed(T * 100 + h)
    rows = 3000
    pool = (torch.randn(rows, 512, generator=g) * 0.5).bfloat16()
    q = (torch.randn(T, h, 512, generator=g) * 0.5).bfloat16()
    idx = torch.randint(0, rows, (T, 128 + 512), generator=g)
    idx[torch.rand(T, 640, generator=g) < 0.3] = -1
    idx[0, :] = -1  # a query with no row gets zeros
    idx[0, 5] = 17 if T > 1 else -1
    idx[-1, 200:] = -1
    sink = torch.randn(h, generator=g) * 2
    scale = 512 ** -0.5
    exp = ref.attend_with_sink(q, pool[idx.clamp_min(0)], idx >= 0, sink, scale)
    got = attend(q.cuda(), pool.cuda(), idx.cuda(), sink.cuda(), scale, splits=splits).cpu()
    assert _rel(got, exp) < 1e-2, _rel(got, exp)
    empty = (idx < 0).all(1)
    assert (got[empty] == 0).all()


@pytest.mark.parametrize("ratio", [1, 2])
def test_core_on_cuda_matches_host(ratio):
    spec = DSv4AttnSpec(heads=16, window=128, ratio=ratio, index_heads=8, index_topk=64, index_heads_per_rank=4,
                        out_groups=2)
    g = torch.Generator().manual_seed(ratio)
    d = 512
    w = dict(freqs=1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64)), sink=torch.randn(16, generator=g),
             comp_norm=(1 + 0.1 * torch.randn(d, generator=g)).bfloat16(),
             wk=(torch.randn(128, d, generator=g) * d ** -0.5).bfloat16(),
             k_norm=(1 + 0.1 * torch.randn(128, generator=g)).bfloat16())
    cores = {dev: DSv4AttnCore(spec, num_slots=2, group_rows=10 * 64, max_step_tokens=320, device=dev,
                               **{k: v.to(dev) for k, v in w.items()}) for dev in ("cpu", "cuda")}
    bt = torch.tensor([[0, 2, 4, 6, 8], [1, 3, 5, 7, 9]])  # 300 positions: up to 300 groups at ratio 1
    n = 300
    inp = dict(q=torch.randn(2, n, 16, d, generator=g).bfloat16(), kv=torch.randn(2, n, d, generator=g).bfloat16(),
               ks=torch.randn(2, n, 2 * d, generator=g), iq=torch.randn(2, n, 8, 128, generator=g).bfloat16(),
               iw=torch.randn(2, n, 8, generator=g).bfloat16())
    done = 0
    for c in [150, 140, 1, 1, 1, 7]:
        seq = torch.tensor([0] * c + [1] * c)
        pos = torch.tensor(list(range(done, done + c)) * 2)
        args = [inp[k][seq, pos] for k in ("q", "kv", "ks", "iq", "iw")]
        if ratio == 1:
            args[2] = None  # ratio 1 compresses the attention's kv row here

        def to(a, dev):
            return None if a is None else a.to(dev)

        out = {dev: cores[dev].step(seq.to(dev), pos.to(dev), torch.tensor([0, 1], device=dev), bt.to(dev),
                                    *[to(a, dev) for a in args]).cpu()
               for dev in ("cpu", "cuda")}
        torch.cuda.synchronize()
        assert _rel(out["cuda"], out["cpu"]) < 2e-2, (c, _rel(out["cuda"], out["cpu"]))
        done += c


@pytest.mark.parametrize("T,H,hpg,N", [(5, 4, 2, 40), (64, 32, 8, 700), (130, 64, 64, 129), (16, 16, 4, 1030)])
def test_index_scores_kernel_matches_rounding_chain(T, H, hpg, N):
    """csrc/dsv4_index.cu against the fp32 statement of the rounding chain (ref.indexer_scores) over the
    same paged keys: almost every score is bit-equal (the fp32 dot products sum in another order, so a
    bf16 rounding may land one ulp apart), and the canonical top-k picks nearly the same groups."""
    from vllm_cmp170hx_b200 import _ext
    from vllm_cmp170hx_b200.oracle import dsv4_attn as ref

    g = torch.Generator().manual_seed(T + H + N)
    nb = (N + 63) // 64
    S = 3
    bt = torch.randperm(S * nb + 5, generator=g)[:S * nb].view(S, nb).to(torch.int32)
    keys = torch.randn((S * nb + 5) * 64, 128, generator=g).bfloat16()
    q = torch.randn(T, H, 128, generator=g).bfloat16()
    w = (torch.randn(T, H, generator=g) * 0.1).bfloat16()
    seq = torch.randint(0, S, (T,), generator=g, dtype=torch.int32)
    n_vis = torch.randint(1, N + 1, (T,), generator=g, dtype=torch.int32)
    gi = torch.arange(N)
    rows = bt[seq.long()][:, gi // 64].long() * 64 + gi % 64
    want = ref.indexer_scores(q, w, keys[rows], n_vis.long(), hpg)
    got = torch.empty(T, N, dtype=torch.float32, device="cuda")
    ops = _ext.ops()
    ops.dsv4_index_scores(q.cuda(), w.cuda(), keys.cuda(), bt.cuda(), seq.cuda(), n_vis.cuda(), hpg, got)
    torch.cuda.synchronize()
    got = got.cpu()
    vis = gi[None] < n_vis[:, None]
    assert torch.equal(torch.isinf(got), ~vis)
    same = (got[vis] == want[vis]).float().mean().item()
    scale = want[vis].abs().max().item()
    print(f"dsv4 index scores: {same:.4f} bit-equal, max diff {(got[vis] - want[vis]).abs().max().item():.2e}")
    assert same > 0.97 and (got[vis] - want[vis]).abs().max().item() <= 0.02 * scale
    k = 16
    top = torch.empty(T, k, dtype=torch.int32, device="cuda")
    cnt = torch.empty(T, dtype=torch.int32, device="cuda")
    ops.mla_topk(want.cuda(), n_vis.cuda(), k, seq.cuda(), bt.cuda(), 64, top, cnt)
    torch.cuda.synchronize()
    sel = ref.select_topk(want, n_vis.long(), k)  # same scores: the same groups, ascending
    rows_ref = torch.where(sel >= 0, rows.gather(1, sel.long().clamp_min(0)), -1)
    assert torch.equal(top.cpu().long(), rows_ref)


@pytest.mark.parametrize("mode,D,heads,norm,inverse", [("fp8", 512, 1, False, False), ("fp8", 512, 8, False, True),
                                                         ("fp4_e4m3", 512, 1, False, False),
                                                         ("fp4_pow2", 128, 4, False, False),
                                                         ("fp4_pow2", 128, 1, True, False),
                                                         ("none", 512, 16, False, False)])
def test_row_transform_kernel_matches_oracle(mode, D, heads, norm, inverse):
    """csrc/dsv4_rot.cu (RMSNorm, RoPE turn in fp64 from fp32 angles, FP8 / FP4 qdq) against the oracle's
    functions: bit-equal except, with the RMSNorm, where the two sums of squares round apart."""
    from vllm_cmp170hx_b200.ops.dsv4_attn import rot_qdq

    g = torch.Generator().manual_seed(D + heads)
    T = 37
    x = (torch.randn(T, heads, D, generator=g) * 3).bfloat16()
    if heads == 1:
        x = x[:, 0]
    pos = torch.randint(-1, 70000, (T,), generator=g)
    freqs = 1.0 / (10000.0 ** (torch.arange(32, dtype=torch.float32) / 32))
    w = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16() if norm else None
    want = rot_qdq(x, pos, freqs, mode, inverse, w, 1e-6).float()
    got = rot_qdq(x.cuda(), pos.cuda(), freqs.cuda(), mode, inverse, None if w is None else w.cuda(), 1e-6)
    torch.cuda.synchronize()
    got = got.cpu().float()
    same = (got == want).float().mean().item()
    print(f"dsv4 row transform {mode}: {same:.4f} bit-equal")
    assert same > (0.99 if norm else 0.999), same
