"""KDA recurrent kernel vs the fp64/fp32 references."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.oracle import kda

pytestmark = pytest.mark.gpu


def test_config1_core_gpu():
    """BASELINE config 1 shapes on the GPU kernel (core mode, fp32 I/O)."""
    g = torch.Generator().manual_seed(0)
    B, T, H, D = 4, 64, 8, 128
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    q, k = q / q.norm(dim=-1, keepdim=True), k / k.norm(dim=-1, keepdim=True)
    gl = torch.nn.functional.logsigmoid(torch.randn(B, T, H, D, generator=g))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    o_ref, S_ref = kda.naive_recurrence(*(x.double() for x in (q, k, v, gl, beta)))
    ops = _ext.ops()
    state = torch.zeros(B, H, D, D, device="cuda")
    has_init = torch.zeros(B, dtype=torch.int32, device="cuda")
    # one decode step per call, state carried in the pool
    outs = []
    for t in range(T):
        cu = torch.arange(0, B + 1, dtype=torch.int32, device="cuda")
        o = torch.empty(B, H, D, device="cuda")
        flat = lambda x: x[:, t].contiguous().cuda()  # noqa: E731
        ops.kda_core(cu, None, has_init, flat(q), flat(k), flat(v), flat(gl), beta[:, t].contiguous().cuda(), state, o)
        has_init.fill_(1)
        outs.append(o.cpu())
    o = torch.stack(outs, dim=1)
    torch.cuda.synchronize()
    assert (o.double() - o_ref).abs().max() < 1e-4
    assert (state.cpu().double() - S_ref).abs().max() < 1e-4


def test_core_prefill_varlen():
    g = torch.Generator().manual_seed(1)
    H, D = 4, 128
    lens = [37, 1, 100]
    T = sum(lens)
    q = torch.randn(T, H, D, generator=g); q = q / q.norm(dim=-1, keepdim=True)
    k = torch.randn(T, H, D, generator=g); k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(T, H, D, generator=g)
    gl = torch.nn.functional.logsigmoid(torch.randn(T, H, D, generator=g))
    beta = torch.sigmoid(torch.randn(T, H, generator=g))
    S0 = torch.randn(3, H, D, D, generator=g) * 0.05
    cu = torch.tensor([0, 37, 38, 138], dtype=torch.int32)
    state = S0.clone().cuda()
    o = torch.empty(T, H, D, device="cuda")
    _ext.ops().kda_core(cu.cuda(), torch.tensor([2, 0, 1], dtype=torch.int32, device="cuda"), None, q.cuda(), k.cuda(),
                        v.cuda(), gl.cuda(), beta.cuda(), state, o)
    for s, slot in enumerate([2, 0, 1]):
        a, b = int(cu[s]), int(cu[s + 1])
        o_ref, S_ref = kda.naive_recurrence(*(x[a:b][None].double() for x in (q, k, v, gl, beta)),
                                            S0[slot][None].double())
        assert (o[a:b].cpu().double() - o_ref[0]).abs().max() < 1e-4
        assert (state[slot].cpu().double() - S_ref[0]).abs().max() < 1e-4


def test_full_layer_semantics():
    """conv + gates + L2 norm + recurrence + gated RMSNorm vs the layer oracle."""
    g = torch.Generator().manual_seed(2)
    H, D = 2, 128
    HD = H * D
    lens = [5, 1, 20]
    T = sum(lens)
    cu = torch.tensor([0, 5, 6, 26], dtype=torch.int32)
    qkv = torch.randn(T, 3 * HD, generator=g).to(torch.bfloat16)
    g_raw = torch.randn(T, HD, generator=g).to(torch.bfloat16)
    beta_raw = torch.randn(T, H, generator=g).to(torch.bfloat16)
    g2 = torch.randn(T, HD, generator=g).to(torch.bfloat16)
    conv_w = (torch.randn(3 * HD, 4, generator=g) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(H, generator=g) * 0.5
    g_bias = torch.randn(HD, generator=g) * 0.1
    norm_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    state = torch.randn(4, H, D, D, generator=g) * 0.05
    conv_state = torch.randn(4, 3 * HD, 3, generator=g).to(torch.bfloat16)
    idx = torch.tensor([3, 1, 0], dtype=torch.int32)
    has_init = torch.tensor([1, 0, 1], dtype=torch.int32)
    st_r, cs_r = state.clone(), conv_state.clone()
    ref = kda.kda_layer(qkv, g_raw, beta_raw, g2, cu, st_r, cs_r, idx, has_init, conv_w, None, a_log, g_bias, -5.0,
                        norm_w)
    st, cs = state.cuda(), conv_state.cuda()
    out = torch.empty(T, HD, dtype=torch.bfloat16, device="cuda")
    _ext.ops().kda_forward(cu.cuda(), idx.cuda(), has_init.cuda(), qkv.cuda(), g_raw.cuda(), beta_raw.cuda(), g2.cuda(),
                           cs, conv_w.cuda(), None, a_log.cuda(), g_bias.cuda(), -5.0, norm_w.cuda(), 1e-5, 1e-6,
                           D ** -0.5, True, st, out)
    torch.cuda.synchronize()
    rel = ((out.cpu().float() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel
    for slot in (3, 1, 0):
        assert (st[slot].cpu() - st_r[slot]).abs().max() < 1e-3
        assert torch.equal(cs[slot].cpu(), cs_r[slot])


def test_verify_records_and_recover_match_prefix():
    """A verify call over k+1 tokens leaves the state untouched; recovering n tokens gives bitwise the
    state (and conv window) of running only those n tokens."""
    from vllm_cmp170hx_b200.ops import kda as kda_ops

    torch.manual_seed(3)
    H, T = 2, 4
    dev = "cuda"
    qkv = (torch.randn(T, 3 * H * 128, device=dev) * 0.5).to(torch.bfloat16)
    g_raw = torch.randn(T, H * 128, device=dev).to(torch.bfloat16)
    beta = torch.randn(T, H, device=dev).to(torch.bfloat16)
    g2 = torch.randn(T, H * 128, device=dev).to(torch.bfloat16)
    conv_w = (torch.randn(3 * H * 128, 4, device=dev) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(H, device=dev)
    norm_w = torch.ones(128, device=dev, dtype=torch.bfloat16)
    st0 = torch.randn(2, H, 128, 128, device=dev) * 0.1
    cv0 = torch.randn(2, 3 * H * 128, 3, device=dev).to(torch.bfloat16)
    cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
    sidx = torch.tensor([1], dtype=torch.int32, device=dev)
    init = torch.ones(1, dtype=torch.int32, device=dev)
    for n in (1, 2, 4):
        st, cv = st0.clone(), cv0.clone()
        recs = kda_ops.KdaRecords()
        kda_ops.kda_forward(qkv, g_raw, beta, g2, cu, sidx, init, cv, conv_w, None, a_log, None, -5.0, norm_w, st,
                            verify=torch.ones(1, dtype=torch.int32, device=dev), records=recs)
        assert torch.equal(st, st0) and torch.equal(cv, cv0)
        kda_ops.kda_recover(recs, torch.tensor([n], dtype=torch.int32), st, cv)
        st_ref, cv_ref = st0.clone(), cv0.clone()
        cu_n = torch.tensor([0, n], dtype=torch.int32, device=dev)
        kda_ops.kda_forward(qkv[:n], g_raw[:n], beta[:n], g2[:n], cu_n, sidx, init, cv_ref, conv_w, None, a_log, None,
                            -5.0, norm_w, st_ref)
        assert torch.equal(st, st_ref), n
        assert torch.equal(cv, cv_ref), n


def _layer_inputs(lens, H, seed, state_scale=0.05):
    g = torch.Generator().manual_seed(seed)
    HD = H * 128
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
    qkv = torch.randn(T, 3 * HD, generator=g).to(torch.bfloat16)
    g_raw = (torch.randn(T, HD, generator=g) * 2).to(torch.bfloat16)
    beta_raw = torch.randn(T, H, generator=g).to(torch.bfloat16)
    g2 = torch.randn(T, HD, generator=g).to(torch.bfloat16)
    conv_w = (torch.randn(3 * HD, 4, generator=g) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(H, generator=g) * 0.5
    g_bias = torch.randn(HD, generator=g) * 0.1
    norm_w = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    S = len(lens)
    state = torch.randn(S + 1, H, 128, 128, generator=g) * state_scale
    conv_state = torch.randn(S + 1, 3 * HD, 3, generator=g).to(torch.bfloat16)
    idx = torch.randperm(S + 1, generator=g)[:S].to(torch.int32)
    has_init = (torch.arange(S) % 2).to(torch.int32)
    return dict(cu=cu, qkv=qkv, g_raw=g_raw, beta_raw=beta_raw, g2=g2, conv_w=conv_w, a_log=a_log, g_bias=g_bias,
                norm_w=norm_w, state=state, conv_state=conv_state, idx=idx, has_init=has_init)


def _run_gpu(x, mode, monkeypatch):
    from vllm_cmp170hx_b200 import envs
    from vllm_cmp170hx_b200.ops import kda as kda_ops

    monkeypatch.setenv("VLLM_B200_KDA_PREFILL", mode)
    envs._cache.clear()
    st, cs = x["state"].cuda(), x["conv_state"].cuda()
    c = {k: v.cuda() for k, v in x.items() if k not in ("state", "conv_state")}
    out = kda_ops.kda_forward(c["qkv"], c["g_raw"], c["beta_raw"], c["g2"], c["cu"], c["idx"], c["has_init"], cs,
                              c["conv_w"], None, c["a_log"], c["g_bias"], -5.0, c["norm_w"], st)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda", 0))
    envs._cache.clear()
    return out.cpu().float(), st.cpu(), cs.cpu()


@pytest.mark.parametrize("lens", [[64], [100, 3, 200, 1, 130], [64, 65, 127, 128, 129], [300]])
def test_chunked_prefill_matches_recurrence(lens, monkeypatch):
    """The chunked tensor-core prefill (sequences of >= 64 tokens; shorter ones stay on the recurrence in
    the same call) against the token recurrence: outputs, final states and conv windows, with fresh and
    continuing sequences, partial last chunks and strong decays (gate pre-activations x2)."""
    H = 4
    x = _layer_inputs(lens, H, seed=len(lens) * 7 + sum(lens))
    o_c, st_c, cs_c = _run_gpu(x, "chunked", monkeypatch)
    o_r, st_r, cs_r = _run_gpu(x, "recurrent", monkeypatch)
    cu = x["cu"].tolist()
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        rel = ((o_c[a:b] - o_r[a:b]).norm() / o_r[a:b].norm()).item()
        slot = int(x["idx"][s])
        ds = (st_c[slot] - st_r[slot]).norm() / st_r[slot].norm()
        print(f"chunked vs recurrence: len {lens[s]} out {rel:.2e} state {ds.item():.2e}")
        assert rel < 2e-2, (s, lens[s], rel)
        assert ds < 1e-2, (s, lens[s], ds.item())
        assert torch.equal(cs_c[slot], cs_r[slot]), s


def test_chunked_prefill_matches_layer_oracle(monkeypatch):
    """One long continuing sequence and one fresh one against the fp32 layer oracle."""
    H = 2
    x = _layer_inputs([150, 70], H, seed=11)
    st_r, cs_r = x["state"].clone(), x["conv_state"].clone()
    ref = kda.kda_layer(x["qkv"], x["g_raw"], x["beta_raw"], x["g2"], x["cu"], st_r, cs_r, x["idx"], x["has_init"],
                        x["conv_w"], None, x["a_log"], x["g_bias"], -5.0, x["norm_w"])
    o_c, st_c, cs_c = _run_gpu(x, "chunked", monkeypatch)
    o_r = _run_gpu(x, "recurrent", monkeypatch)[0]
    rel = ((o_c - ref).norm() / ref.norm()).item()
    rel_r = ((o_r - ref).norm() / ref.norm()).item()
    print(f"vs layer oracle: chunked {rel:.2e} recurrent {rel_r:.2e}")
    assert rel < 2e-2, rel
    for s in range(2):
        slot = int(x["idx"][s])
        assert ((st_c[slot] - st_r[slot]).norm() / st_r[slot].norm()).item() < 1e-2
