"""DFlash block drafter on CPU: the paged context cache and the non-causal block forward against a
dense fp32 restatement, and greedy speculative decoding with DFlash drafts emitting exactly the
tokens of plain greedy decoding (reference drafter shape: upstream qwen3_dflash via
vllm_sm80/spec_decode/dflash_draft.py)."""

import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_deepseek
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.dflash import DFlashConfig, DFlashDrafter
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _cfg(k=0, method="mtp"):
    return EngineConfig(model=tiny_deepseek(layers=3, experts=4, hidden=256, vocab=512),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256,
                                                  num_speculative_tokens=k, spec_method=method),
                        cache=CacheConfig(num_blocks=48), device="cpu", enforce_eager=True)


def _rms(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()


def _rope(x, pos, theta):
    hd = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2).float() / hd))
    ang = pos.float()[:, None, None] * inv
    a, b = x[..., : hd // 2], x[..., hd // 2:]
    return torch.cat([a * ang.cos() - b * ang.sin(), b * ang.cos() + a * ang.sin()], -1)


def _dense_block(d: DFlashDrafter, target, states, bonus, k):
    """Dense fp32 restatement for ONE request: context states [C, H] at positions 0..C-1."""
    dc, L = d.dc, d.layers[0]
    C = states.shape[0]
    nh, nkv, hd, eps = dc.num_heads, dc.num_kv_heads, dc.head_dim, L.input_norm.eps
    ctx = _rms(states, d.hidden_norm.weight, eps)
    ids = torch.tensor([bonus] + [dc.mask_token_id] * k)
    pos = torch.arange(C, C + k + 1)
    x = target.embed[ids].float()
    res = None
    for L in d.layers:
        W = L.qkv.weight.float()
        kc = (ctx @ W[nh * hd:(nh + nkv) * hd].t()).view(C, nkv, hd)
        vc = (ctx @ W[(nh + nkv) * hd:].t()).view(C, nkv, hd)
        kc = _rope(_rms(kc, L.k_norm.weight, eps), torch.arange(C), dc.rope_theta)
        res = x if res is None else res + x
        h = _rms(res, L.input_norm.weight, eps)
        q, kb, vb = (h @ W.t()).split([nh * hd, nkv * hd, nkv * hd], -1)
        q = _rope(_rms(q.view(-1, nh, hd), L.q_norm.weight, eps), pos, dc.rope_theta)
        kb = _rope(_rms(kb.view(-1, nkv, hd), L.k_norm.weight, eps), pos, dc.rope_theta)
        K = torch.cat([kc, kb], 0).repeat_interleave(nh // nkv, 1)
        V = torch.cat([vc, vb.view(-1, nkv, hd)], 0).repeat_interleave(nh // nkv, 1)
        att = torch.einsum("qhd,khd->hqk", q, K) * hd ** -0.5
        o = torch.einsum("hqk,khd->qhd", att.softmax(-1), V).reshape(-1, nh * hd)
        a = o @ L.o_proj.weight.float().t()
        res = res + a
        h = _rms(res, L.post_norm.weight, eps)
        g, u = (h @ L.gate_up.weight.float().t()).chunk(2, -1)
        x = (torch.nn.functional.silu(g) * u) @ L.down.weight.float().t()
    return _rms(res + x, d.norm.weight, eps)[1:]


def test_block_forward_over_paged_context_matches_dense():
    pstate.set_state(pstate.ParallelState())
    cfg = _cfg().model
    target = HybridForCausalLM(cfg, "cpu", seed=1)
    d = DFlashDrafter(cfg, DFlashConfig(num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64, intermediate=256),
                      target, "cpu", seed=2)
    caches = d.alloc_caches(8 * 64, "cpu")
    g = torch.Generator().manual_seed(0)
    lens, blocks = [70, 33], [[5, 2], [7]]
    states = [torch.randn(n, 256, generator=g).bfloat16() for n in lens]
    for st, n, b in zip(states, lens, blocks):
        p = torch.arange(n)
        slots = torch.tensor(b)[p // 64] * 64 + p % 64
        d.store_context(st, p, slots, caches)
    C = max(lens)
    cs = torch.full((2, C), -1, dtype=torch.long)
    for a, (n, b) in enumerate(zip(lens, blocks)):
        p = torch.arange(n)
        cs[a, :n] = torch.tensor(b)[p // 64] * 64 + p % 64
    k = 3
    h = d(torch.tensor([11, 22]), torch.tensor(lens) - 1, cs, cs >= 0, caches, k)
    d.gather_bytes = 1  # one request per group: the same rows
    assert torch.equal(d(torch.tensor([11, 22]), torch.tensor(lens) - 1, cs, cs >= 0, caches, k), h)
    for a in range(2):
        exp = _dense_block(d, target, states[a], [11, 22][a], k)
        err = ((h[a].float() - exp).norm() / exp.norm()).item()
        assert err < 3e-2, (a, err)


def test_greedy_dflash_spec_matches_plain():
    pstate.set_state(pstate.ParallelState())
    prompts = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]
    model = HybridForCausalLM(_cfg().model, "cpu", seed=3)
    plain = LLM(_cfg(), model).generate(prompts, SamplingParams(max_tokens=8))
    llm = LLM(_cfg(k=3, method="dflash"), model)
    spec = llm.generate(prompts, SamplingParams(max_tokens=8))
    assert [o.output_token_ids for o in spec] == [o.output_token_ids for o in plain]
    sd = llm.engine.runner.spec
    assert sd.method == "dflash" and sd.stats["proposed"] > 0
    assert model.aux_layer_ids and len(model.aux_hidden) == len(model.aux_layer_ids)
    model.aux_layer_ids = ()
