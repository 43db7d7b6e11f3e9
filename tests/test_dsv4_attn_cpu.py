"""DeepSeek-V4.1 attention core on the host: the quantize-dequantize grids, and the cached,
chunked core (window ring, compressed groups at ratio 1 and 2, indexer top-k, candidate blocks,
sinks) against a from-scratch per-token recomputation (reference: models/deepseek_v41/ops/
sm80_attn_core.py, ops/sm80_act_quant.py)."""

import pytest
import torch

from vllm_cmp170hx_b200.oracle import dsv4_attn as ref
from vllm_cmp170hx_b200.ops.dsv4_attn import DSv4AttnCore, DSv4AttnSpec


def test_qdq_grids():
    x = torch.tensor([[0.0, 0.3, -1.1, 2.6, 5.0, -6.0, 100.0, 7e-3] * 4])
    y = ref.fp4_qdq(x, 32, "pow2")
    s = 32.0  # the smallest power of two >= 100 / 6
    grid = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6])
    q = (y / s).abs().flatten()
    assert all(bool((grid == v).any()) for v in q), q
    y8 = ref.fp8_qdq(x, 32)
    assert torch.equal(y8, ref.fp8_qdq(y8, 32))  # values on the grid stay put
    assert ((y8 - x).abs() <= x.abs() * 2 ** -3 + 2 ** -9 * 2 ** -2).all()
    # e4m3 block scales: s = e4m3(amax / 6)
    z = ref.fp4_qdq(torch.full((1, 16), 0.75), 16, "e4m3")
    assert torch.allclose(z, torch.full((1, 16), 0.75))


def _weights(spec, seed=0):
    g = torch.Generator().manual_seed(seed)
    d = spec.head_dim
    freqs = 1.0 / (10000 ** (torch.arange(0, spec.rope_dim, 2).float() / spec.rope_dim))
    return dict(freqs=freqs, sink=torch.randn(spec.heads, generator=g),
                comp_norm=(1 + 0.1 * torch.randn(d, generator=g)).bfloat16(),
                wk=(torch.randn(spec.index_dim, d, generator=g) * d ** -0.5).bfloat16(),
                k_norm=(1 + 0.1 * torch.randn(spec.index_dim, generator=g)).bfloat16())


def _inputs(spec, n, seed):
    g = torch.Generator().manual_seed(seed)
    d = spec.head_dim
    return dict(q=torch.randn(n, spec.heads, d, generator=g).bfloat16(),
                kv=torch.randn(n, d, generator=g).bfloat16(),
                ks=torch.randn(n, 2 * d, generator=g),
                iq=torch.randn(n, spec.index_heads, spec.index_dim, generator=g).bfloat16(),
                iw=torch.randn(n, spec.index_heads, generator=g).bfloat16())


def _scratch(spec, w, inp, p, cand=None):
    """Query at position p of one sequence, recomputed from the raw inputs of positions 0..p."""
    fr = w["freqs"]
    pos = torch.tensor([p])
    rows, valid = [], []
    for b in range(spec.window):
        j = p - b
        ok = j >= 0
        rows.append(ref.window_kv(inp["kv"][max(j, 0)][None], torch.tensor([max(j, 0)]), fr)[0])
        valid.append(ok)
    n_vis = (p + 1) // spec.ratio
    sel = torch.full((spec.index_topk,), -1)
    comp = []
    if n_vis:
        lat, gpos = [], []
        for gi in range(n_vis):
            if spec.ratio == 1:
                lat.append(ref.rms_norm(inp["kv"][gi][None], w["comp_norm"], spec.eps)[0])
            else:
                lat.append(ref.pooled_pair(inp["ks"][2 * gi][None], inp["ks"][2 * gi + 1][None], w["comp_norm"],
                                         spec.eps)[0])
            gpos.append(gi * spec.ratio)
        lat, gpos = torch.stack(lat), torch.tensor(gpos)
        comp = ref.compressed_kv(lat, gpos, fr)
        keys = ref.index_key((lat.float() @ w["wk"].float().t()).bfloat16(), w["k_norm"], gpos, fr, spec.eps)
        qi = ref.index_q(inp["iq"][p][None], pos, fr)
        wi = (inp["iw"][p][None].float() * (spec.index_dim ** -0.5 * spec.index_heads ** -0.5)).bfloat16()
        sc = ref.indexer_scores(qi, wi, keys[None], torch.tensor([n_vis]), spec.index_heads_per_rank)
        if cand is not None:
            sc = ref.restrict_to_blocks(sc, cand[None], spec.candidate_block)
        sel = ref.select_topk(sc, torch.tensor([n_vis]), spec.index_topk)[0]
        cb = ref.pick_blocks(sc, torch.tensor([n_vis]), spec.candidate_blocks, spec.candidate_block)[0] \
            if spec.candidate_blocks else None
    else:
        cb = torch.full((spec.candidate_blocks,), -1, dtype=torch.int32) if spec.candidate_blocks else None
    for s in sel.tolist():
        rows.append(comp[s] if s >= 0 else torch.zeros(spec.head_dim, dtype=torch.bfloat16))
        valid.append(s >= 0)
    qr = ref.rotate(inp["q"][p][None], pos, fr)
    o = ref.attend_with_sink(qr, torch.stack(rows)[None], torch.tensor(valid)[None], w["sink"], spec.head_dim ** -0.5)
    return ref.finish_output(o, pos, fr)[0], cb


def _run(spec, w, seqs, chunks, device="cpu", candidates=None):
    """Two interleaved sequences stepped through the core in the given chunk sizes."""
    core = DSv4AttnCore(spec, num_slots=3, group_rows=4 * 64, max_step_tokens=2 * max(chunks), device=device, **w)
    bt = torch.tensor([[3], [1]], device=device)  # one 64-row block per sequence, not in order
    slot = torch.tensor([2, 0], device=device)
    done = [0, 0]
    outs = [[None] * len(s["kv"]) for s in seqs]
    cands = [[None] * len(s["kv"]) for s in seqs]
    for c in chunks:
        seq, pos = [], []
        for s in range(2):
            n = min(c, len(seqs[s]["kv"]) - done[s])
            seq += [s] * n
            pos += list(range(done[s], done[s] + n))
        if not seq:
            break
        seq_t, pos_t = torch.tensor(seq), torch.tensor(pos)

        def pick(key):
            return torch.stack([seqs[s][key][p] for s, p in zip(seq, pos)]).to(device)
        cin = None
        if candidates is not None:
            cin = torch.stack([candidates[s][p] for s, p in zip(seq, pos)]).to(device)
        cout = []
        ks = pick("ks") if spec.ratio == 2 else None  # ratio 1 compresses the attention's kv row here
        o = core.step(seq_t.to(device), pos_t.to(device), slot, bt, pick("q"), pick("kv"), ks, pick("iq"),
                      pick("iw"),
                      candidates_in=cin, candidates_out=cout if spec.candidate_blocks else None)
        for i, (s, p) in enumerate(zip(seq, pos)):
            outs[s][p] = o[i].cpu()
            if cout:
                cands[s][p] = cout[0][i].cpu()
        for s in range(2):
            done[s] += seq.count(s)
    return outs, cands


@pytest.mark.parametrize("ratio", [1, 2])
def test_chunked_core_matches_from_scratch(ratio):
    spec = DSv4AttnSpec(heads=4, window=8, ratio=ratio, index_heads=4, index_topk=5, index_heads_per_rank=2,
                        out_groups=2)
    w = _weights(spec)
    seqs = [_inputs(spec, 23, 1), _inputs(spec, 17, 2)]
    outs, _ = _run(spec, w, seqs, [6, 5, 1, 1, 4, 1, 1, 7, 1, 1])
    for s in range(2):
        for p in range(len(seqs[s]["kv"])):
            exp, _ = _scratch(spec, w, seqs[s], p)
            assert torch.equal(outs[s][p], exp), (ratio, s, p)


def test_candidate_blocks_two_levels():
    """A source layer picks candidate blocks; a user layer attends only inside them."""
    src = DSv4AttnSpec(heads=2, window=4, ratio=1, index_heads=2, index_topk=6, index_heads_per_rank=2,
                       candidate_blocks=2, candidate_block=4)
    w = _weights(src, 3)
    seqs = [_inputs(src, 30, 4), _inputs(src, 21, 5)]
    _, cands = _run(src, w, seqs, [9, 1, 1, 12, 1, 1, 9])
    for s in range(2):
        for p in range(len(seqs[s]["kv"])):
            _, cb = _scratch(src, w, seqs[s], p)
            assert torch.equal(cands[s][p], cb), (s, p)
    user = DSv4AttnSpec(heads=2, window=4, ratio=1, index_heads=2, index_topk=3, index_heads_per_rank=2,
                        candidate_block=4)
    outs, _ = _run(user, w, seqs, [9, 1, 1, 12, 1, 1, 9], candidates=cands)
    for s in range(2):
        for p in range(len(seqs[s]["kv"])):
            exp, _ = _scratch(user, w, seqs[s], p, cand=cands[s][p])
            assert torch.equal(outs[s][p], exp), (s, p)


def test_e2m1_nearest_ties_to_even_code():
    """Every magnitude on a fine grid (thresholds included) goes to the nearest E2M1 value; on a tie
    the value with the even code (0, 1, 2, 4) wins."""
    grid = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    xs = torch.arange(0, 6.0001, 1 / 64)
    got = ref.e2m1(torch.cat([xs, -xs]))
    for i, x in enumerate(xs.tolist()):
        d = [abs(x - g) for g in grid]
        best = min(d)
        cands = [c for c, v in enumerate(d) if v == best]
        code = cands[0] if len(cands) == 1 else [c for c in cands if c % 2 == 0][0]
        assert got[i].item() == grid[code], x
        assert got[len(xs) + i].item() == -grid[code], x


def test_selection_against_sorted_pairs():
    """select_topk / pick_blocks against a plain sort of (-score, column) pairs, with repeated scores,
    signed zeros and -FLT_MAX entries."""
    g = torch.Generator().manual_seed(7)
    n, N, k = 6, 40, 9
    scores = torch.randint(-3, 4, (n, N), generator=g).float()
    scores[scores == 0] = torch.tensor(-0.0)
    scores[:, ::7] = 0.0
    scores[1, 3:20] = ref.NEG_FLT_MAX
    n_vis = torch.tensor([40, 5, 9, 1, 0, 23])
    scores = torch.where(torch.arange(N)[None] < n_vis[:, None], scores, float("-inf"))
    got = ref.select_topk(scores, n_vis, k)
    for i in range(n):
        pairs = sorted((-scores[i, c].item(), c) for c in range(int(n_vis[i])))
        want = sorted(c for _, c in pairs[:k])
        assert got[i].tolist() == want + [-1] * (k - len(want)), i
    blk = 4
    got_b = ref.pick_blocks(scores, n_vis, 3, blk)
    for i in range(n):
        nv = int(n_vis[i])
        nb = -(-nv // blk)
        best = [max(scores[i, b * blk:min(N, b * blk + blk)].tolist()) for b in range(nb)]
        if nv:
            best[(nv - 1) // blk] = float("inf")
        pairs = sorted((-(v + 0.0), b) for b, v in enumerate(best))
        want = sorted(b for _, b in pairs[:3])
        assert got_b[i].tolist() == want + [-1] * (3 - len(want)), i


def test_indexer_score_rounding_chain():
    """indexer_scores against a scalar evaluation of the stated rounding chain."""
    import numpy as np

    g = torch.Generator().manual_seed(3)
    H, D, N, hpg = 8, 16, 5, 4
    q = torch.randn(2, H, D, generator=g).bfloat16()
    w = torch.randn(2, H, generator=g).bfloat16()
    keys = torch.randn(2, N, D, generator=g).bfloat16()
    got = ref.indexer_scores(q, w, keys, torch.tensor([N, 3]), hpg)

    def bf(x):
        return float(torch.tensor(x, dtype=torch.float32).bfloat16().float())

    for i in range(2):
        for c in range(N):
            if c >= [N, 3][i]:
                assert got[i, c].item() == float("-inf")
                continue
            total = None
            for r in range(H // hpg):
                acc = np.float32(0)
                for h in range(r * hpg, (r + 1) * hpg):
                    dot = float(np.dot(q[i, h].float().double().numpy(), keys[i, c].float().double().numpy()))
                    t = bf(float(np.float32(w[i, h].float().item()) * np.float32(max(bf(dot), 0.0))))
                    acc = np.float32(acc + np.float32(t)) if h > r * hpg else np.float32(t)
                part = bf(float(acc))
                total = part if total is None else bf(float(np.float32(total) + np.float32(part)))
            assert got[i, c].item() == total, (i, c)
