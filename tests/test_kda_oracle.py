"""KDA gated-delta-rule decode correctness on CPU.

fp32, batch 4, 8 heads, head_dim_k = head_dim_v = 128, 64 sequential decode
steps from a zero state; q, k, v ~ N(0, 1) seeded, q and k L2-normalised per
head; per-channel decay g = logsigmoid(N(0, 1)); beta = sigmoid(N(0, 1)).
The engine's CPU path (chunk-parallel form) and a token-by-token decode loop
(one call per step, state carried) are checked against the naive recurrence.
"""

import torch

from vllm_cmp170hx_b200.oracle import kda


def _inputs(dtype=torch.float32, B=4, T=64, H=8, D=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    gl = torch.nn.functional.logsigmoid(torch.randn(B, T, H, D, generator=g))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    return [x.to(dtype) for x in (q, k, v, gl, beta)]


def test_config1_chunked_matches_naive():
    q, k, v, g, beta = _inputs(torch.float64)
    o_ref, S_ref = kda.naive_recurrence(q, k, v, g, beta)
    for chunk in (64, 16, 7):
        o, S = kda.chunked(q, k, v, g, beta, chunk=chunk)
        assert torch.allclose(o, o_ref, atol=1e-10, rtol=1e-9), chunk
        assert torch.allclose(S, S_ref, atol=1e-10, rtol=1e-9), chunk


def test_config1_fp32_step_by_step_decode():
    q, k, v, g, beta = _inputs(torch.float32)
    o_ref, S_ref = kda.naive_recurrence(*(x.double() for x in (q, k, v, g, beta)))
    S = None
    outs = []
    for t in range(q.shape[1]):
        o, S = kda.chunked(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1], S)
        outs.append(o)
    o = torch.cat(outs, dim=1)
    assert (o.double() - o_ref).abs().max() < 1e-4
    assert (S.double() - S_ref).abs().max() < 1e-4


def test_chunked_with_initial_state():
    q, k, v, g, beta = _inputs(torch.float64, B=2, T=40, H=2)
    S0 = torch.randn(2, 2, 128, 128, dtype=torch.float64) * 0.1
    o_ref, S_ref = kda.naive_recurrence(q, k, v, g, beta, S0)
    o, S = kda.chunked(q, k, v, g, beta, S0, chunk=16)
    assert torch.allclose(o, o_ref, atol=1e-10) and torch.allclose(S, S_ref, atol=1e-10)
