"""Speculative decoding on CPU (oracle kernels): MTP drafter + verification.

Greedy speculative decoding must emit exactly the tokens of plain greedy
decoding whatever the drafts are (random MTP weights: mostly rejected;
oracle drafts: all accepted, bonus token every step; half-wrong drafts), and
rejection sampling must leave the target distribution unchanged.
"""

import types

import numpy as np
import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_deepseek
from vllm_cmp170hx_b200.engine import spec_decode
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import Request, SamplingParams
from vllm_cmp170hx_b200.engine.scheduler import ScheduledReq, SchedulerOutput
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _cfg(k=0, budget=64):
    return EngineConfig(model=tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=budget, max_model_len=256,
                                                  num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=48), device="cpu", enforce_eager=True)


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg().model, "cpu", seed=3)


PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]
MAX_TOKENS = [12, 9, 7]


def _plain(model):
    params = [SamplingParams(max_tokens=m) for m in MAX_TOKENS]
    return [o.output_token_ids for o in LLM(_cfg(), model).generate(PROMPTS, params)]


def test_greedy_spec_matches_plain(model):
    ref = _plain(model)
    params = [SamplingParams(max_tokens=m) for m in MAX_TOKENS]
    llm = LLM(_cfg(k=3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, params)]
    assert got == ref
    assert llm.engine.runner.spec.stats["proposed"] > 0


@pytest.mark.parametrize("mode", ["oracle", "half"])
def test_greedy_spec_with_planted_drafts(model, mode, monkeypatch):
    ref = _plain(model)
    by_prompt = {tuple(p): r for p, r in zip(PROMPTS, ref)}

    def fake_propose(self, out, hidden, accepted):
        for s in out.reqs:
            req = s.req
            if req.status.finished or req.num_computed_tokens != req.num_tokens - 1:
                continue
            full = by_prompt[tuple(req.prompt_token_ids)]
            n = len(req.output_token_ids)
            d = list(full[n:n + self.k])
            if mode == "half":
                d = [t if (i % 2 == 0) else (t + 1) % 512 for i, t in enumerate(d)]
            limit = max(0, min(self.k, req.params.max_tokens - n - 1))
            req.draft_token_ids = d[:limit]

    monkeypatch.setattr(spec_decode.SpecDecoder, "propose", fake_propose)
    params = [SamplingParams(max_tokens=m) for m in MAX_TOKENS]
    llm = LLM(_cfg(k=3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, params)]
    assert got == ref
    st = llm.engine.runner.spec.stats
    if mode == "oracle":
        assert st["accepted"] == st["proposed"] > 0
        # every verify step yields k+1 tokens, so far fewer steps than tokens
        assert llm.engine.num_steps < sum(MAX_TOKENS)
    else:
        assert 0 < st["accepted"] < st["proposed"]


def test_sampled_spec_runs(model):
    params = [SamplingParams(max_tokens=m, temperature=0.7) for m in MAX_TOKENS]
    llm = LLM(_cfg(k=2), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, params)]
    assert [len(g) for g in got] == MAX_TOKENS
    assert all(0 <= t < 512 for g in got for t in g)


def test_rejection_sampling_preserves_target_distribution():
    """One draft from q, verified against p: the emitted first token is distributed as p."""
    pstate.set_state(pstate.ParallelState())
    V = 6
    rng = np.random.default_rng(0)
    p_logits = torch.tensor(rng.normal(size=V) * 1.5, dtype=torch.float32)
    q = torch.softmax(torch.tensor(rng.normal(size=V), dtype=torch.float32), -1)
    T = 1.0
    p = torch.softmax(p_logits / T, -1)
    runner = types.SimpleNamespace(model=types.SimpleNamespace(vocab_offset=0),
                                   cfg=types.SimpleNamespace(seed=11), step_counter=torch.zeros(1, dtype=torch.int64))
    dec = spec_decode.SpecDecoder.__new__(spec_decode.SpecDecoder)
    dec.runner, dec.k, dec.step_no, dec.q_store = runner, 1, 0, {}
    dec.stats = {"proposed": 0, "accepted": 0, "steps": 0}
    g = torch.Generator().manual_seed(5)
    N = 6000
    counts = np.zeros(V)
    logits = torch.stack([p_logits, p_logits])  # row 0 verifies the draft, row 1 is the bonus row
    for it in range(N):
        d = int(torch.multinomial(q, 1, generator=g))
        req = Request([1, 2, 3], SamplingParams(max_tokens=4, temperature=T), request_id="r")
        req.output_token_ids = [4]
        req.draft_token_ids = [d]
        dec.q_store["r"] = (q.view(1, 1, V), 0)
        out = SchedulerOutput(reqs=[ScheduledReq(req, 2, 3, True, 1)])
        res = dec.verify(out, logits, {"r": [0, 1]})
        runner.step_counter += 1
        counts[res["r"][0]] += 1
    emp = counts / N
    assert np.abs(emp - p.numpy()).max() < 0.025, (emp, p.numpy())


def test_adaptive_k_policies():
    from vllm_cmp170hx_b200.engine.adaptive_k import AdaptiveKPolicy, expected_tokens

    p = AdaptiveKPolicy(3)
    assert [p.choose(n) for n in (1, 8, 20, 100, 1000)] == [3, 3, 2, 1, 1]
    assert abs(expected_tokens(3, 0.5) - 1.875) < 1e-9 and expected_tokens(2, 1.0) == 3
    a = AdaptiveKPolicy(3, mode="accept")
    a.accept_rate = 0.9
    assert a.choose(1) == 3  # cheap drafts, high acceptance: full depth
    a.accept_rate = 0.05
    for _ in range(3):
        k = a.choose(400)  # compute-bound batch, drafts rarely accepted: no drafts
    assert k == 0


def test_greedy_spec_with_adaptive_k_matches_plain(model):
    ref = _plain(model)
    cfg = _cfg(k=3)
    cfg.scheduler.adaptive_k = "by_load"
    llm = LLM(cfg, model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, [SamplingParams(max_tokens=m) for m in MAX_TOKENS])]
    assert got == ref and llm.engine.scheduler.draft_cap == 3


def _hybrid_cfg(k=0):
    from vllm_cmp170hx_b200.config import tiny

    m = tiny(layers=4, experts=4, expert_format="bf16", layer_types=["kda", "mla", "kda", "kda"])
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256,
                                                           num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=48), device="cpu", enforce_eager=True)


@pytest.mark.parametrize("mode", ["mtp", "oracle", "half"])
def test_hybrid_kda_spec_matches_plain(mode, monkeypatch):
    """Speculative decoding through KDA layers: the verify step records the recurrence updates and
    the recovery applies only the accepted prefix, so greedy output equals plain decoding."""
    pstate.set_state(pstate.ParallelState())
    m = HybridForCausalLM(_hybrid_cfg().model, "cpu", seed=6)
    params = [SamplingParams(max_tokens=n) for n in MAX_TOKENS]
    ref = [o.output_token_ids for o in LLM(_hybrid_cfg(), m).generate(PROMPTS, params)]
    if mode != "mtp":
        by_prompt = {tuple(p): r for p, r in zip(PROMPTS, ref)}

        def planted(self, out, hidden, accepted):
            for s in out.reqs:
                req = s.req
                if req.status.finished or req.num_computed_tokens != req.num_tokens - 1:
                    continue
                n = len(req.output_token_ids)
                d = list(by_prompt[tuple(req.prompt_token_ids)][n:n + self.k])
                if mode == "half":
                    d = [t if i % 2 == 0 else (t + 1) % 500 for i, t in enumerate(d)]
                req.draft_token_ids = d[:max(0, min(self.k, req.params.max_tokens - n - 1))]

        monkeypatch.setattr(spec_decode.SpecDecoder, "propose", planted)
    llm = LLM(_hybrid_cfg(k=3), m)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, params)]
    assert got == ref
    st = llm.engine.runner.spec.stats
    assert st["proposed"] > 0
    if mode == "oracle":
        assert st["accepted"] == st["proposed"]
