"""Qwen3-Next-style family on CPU: the gated delta net against a scalar-decay recurrence written from its
definition, the gated attention ops against whole-prompt attention, n-gram ids against a direct hash,
and the model in the engine (generation independent of prompt chunking, greedy MTP speculative decoding
equal to plain decoding)."""

import numpy as np
import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_qwen
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.models.qwen import ngram_ids
from vllm_cmp170hx_b200.ops import gqa as gqa_ops
from vllm_cmp170hx_b200.oracle import gqa as gqa_ref
from vllm_cmp170hx_b200.oracle import kda as kda_ref
from vllm_cmp170hx_b200.oracle.mla import rope_cos_sin
from vllm_cmp170hx_b200.parallel import state as pstate


def test_gdn_gate_mode_matches_scalar_recurrence():
    torch.manual_seed(0)
    H, D, T = 2, 128, 7
    qkv = torch.randn(T, 3 * H * D)
    a = torch.randn(T, H)
    b = torch.randn(T, H)
    z = torch.randn(T, H * D)
    a_log = torch.randn(H) * 0.3
    dt_bias = torch.randn(H) * 0.3
    norm_w = 1 + 0.1 * torch.randn(D)
    state = torch.zeros(1, H, D, D)
    conv_state = torch.zeros(1, 3 * H * D, 3)
    cu = torch.tensor([0, T], dtype=torch.int32)
    conv_w = torch.zeros(3 * H * D, 4)
    conv_w[:, 3] = 1.0  # identity taps: the conv + SiLU is SiLU
    out = kda_ref.kda_layer(qkv, a, b, z, cu, state, conv_state, None, None, conv_w, None, a_log, dt_bias, 0.0,
                            norm_w, eps=1e-6, round_conv=False, gate_mode=1)
    # definition: per head one decay alpha_t = exp(-exp(A) softplus(a_t + dt)), S <- alpha S + beta (v - S k) k^T
    act = torch.nn.functional.silu(qkv)
    q = act[:, :H * D].view(T, H, D)
    k = act[:, H * D:2 * H * D].view(T, H, D)
    v = act[:, 2 * H * D:].view(T, H, D)
    ref = torch.zeros(T, H, D)
    for h in range(H):
        S = torch.zeros(D, D, dtype=torch.float64)
        for t in range(T):
            qt = q[t, h].double() / q[t, h].double().norm() * D ** -0.5
            kt = k[t, h].double() / k[t, h].double().norm()
            alpha = torch.exp(-torch.exp(a_log[h].double()) * torch.nn.functional.softplus(a[t, h].double() +
                                                                                          dt_bias[h].double()))
            beta = torch.sigmoid(b[t, h].double())
            S = alpha * S
            S = S + beta * torch.outer(v[t, h].double() - S @ kt, kt)
            o = S @ qt
            o = o / torch.sqrt((o * o).mean() + 1e-6) * norm_w.double()
            ref[t, h] = (o * torch.nn.functional.silu(z[t, h * D:(h + 1) * D].double())).float()
    assert torch.allclose(out.view(T, H, D), ref, atol=2e-4, rtol=1e-4)


def test_gqa_ops_match_whole_prompt_attention():
    torch.manual_seed(1)
    nh, nkv, T1, T2 = 4, 2, 5, 9
    T = T1 + T2
    proj = (torch.randn(T, nh * 512 + nkv * 512) * 0.5).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(256)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(256)).to(torch.bfloat16)
    cs = rope_cos_sin(64, 64, 1e7)
    pos = torch.tensor(list(range(T1)) + list(range(T2)), dtype=torch.int32)
    # two sequences in blocks 1 and 0 of a 2-block cache
    bt = torch.tensor([[1], [0]], dtype=torch.int32)
    tseq = torch.tensor([0] * T1 + [1] * T2, dtype=torch.int32)
    slots = (bt[tseq.long(), 0].long() * 64 + pos.long())
    cache = torch.zeros(2 * 64 * nkv, 512, dtype=torch.bfloat16)
    q = torch.empty(T * nkv, nh // nkv, 512, dtype=torch.bfloat16)
    gqa_ops.prep(proj, nh, nkv, qw, kw, 1e-6, pos, cs, slots, q, cache)
    o = gqa_ops.attention(q, cache, pos + 1, tseq, bt, nkv, T2)
    y = gqa_ops.gate(o, proj, nh)
    ref = gqa_ref.layer_core(proj, nh, nkv, qw, kw, 1e-6, pos, cs, [0, T1], [T1, T2])
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2)


def test_ngram_ids_match_direct_hash():
    toks = np.array([7, 3, 9, 11, 2], dtype=np.int64)
    offs, voc, mult = np.array([0, 100]), np.array([100, 50]), np.array([1000003, 7, 13, 17])
    got = ngram_ids(toks, np.arange(5), [2, 3], offs, voc, mult)
    for p in range(5):
        for h, n in enumerate([2, 3]):
            key = 0
            for i in range(n):
                t = toks[p - i] + 1 if p - i >= 0 else 0
                key += t * int(mult[(h + i) % 4])
            assert got[p, h] == offs[h] + key % voc[h]


PROMPTS = [[(7 * i + 5 * j) % 500 for j in range(n)] for i, n in enumerate([11, 37, 70])]


def _cfg(budget, k=0):
    m = tiny_qwen(layers=4)
    m.num_mtp_layers = 1 if k else 0
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=budget,
                                                           max_model_len=256, num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg(32).model, "cpu", seed=11)


def _gen(model, cfg, n=6):
    return [o.output_token_ids for o in LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=n))]


def test_qwen_generation_independent_of_chunking(model):
    a = _gen(model, _cfg(16))
    b = _gen(model, _cfg(128))
    assert a == b and all(len(x) == 6 for x in a)


def test_qwen_greedy_mtp_spec_matches_plain(model):
    plain = _gen(model, _cfg(64))
    llm = LLM(_cfg(64, k=2), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, SamplingParams(max_tokens=6))]
    assert got == plain
    assert llm.engine.runner.spec.stats["proposed"] > 0
