"""DeepSeek-family model and MTP speculative decoding on the GPU: the tiny
DeepSeek model (fp8 block-scaled attention projections, Marlin int4 experts)
against the CPU oracle, and greedy speculative decoding against plain greedy
decoding (CUDA-graph decode)."""

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_deepseek
from vllm_cmp170hx_b200.engine import spec_decode
from vllm_cmp170hx_b200.engine.llm_engine import LLM, LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate

pytestmark = pytest.mark.gpu


def _cfg(device, k=0, eager=False):
    return EngineConfig(model=tiny_deepseek(layers=3, experts=8, hidden=256, vocab=512),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                                                  num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=40), device=device, enforce_eager=eager,
                        cuda_graph_batch_sizes=[1, 2, 4])


PROMPTS = [list(range(3, 3 + n)) for n in (12, 70, 131)]
MAX_TOKENS = [10, 8, 7]


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg("cuda").model, "cuda", seed=9)


def test_deepseek_forward_matches_cpu_oracle():
    pstate.set_state(pstate.ParallelState())
    logits = {}
    for dev in ("cpu", "cuda"):
        cfg = _cfg(dev, eager=True)
        # every position and every expert selected: compares arithmetic, not near-tie selections
        # (a router near-tie flips one token's experts between the two paths otherwise)
        cfg.model.mla.index_topk = 128
        cfg.model.moe.top_k = cfg.model.moe.num_experts
        m = HybridForCausalLM(cfg.model, dev, seed=3, init_mode="sliced")
        eng = LLMEngine(cfg, m)
        for p in PROMPTS[:2]:
            eng.add_request(p, SamplingParams(max_tokens=1))
        out = eng.scheduler.schedule()
        h = eng.runner._host_inputs(out)
        d, ctx, _ = eng.runner._context(h)
        with torch.inference_mode():
            logits[dev] = m.compute_logits(m(d["ids"], ctx)).float().cpu()
    rel = ((logits["cuda"] - logits["cpu"]).norm() / logits["cpu"].norm()).item()
    assert rel < 5e-2, rel


def _plain(model):
    params = [SamplingParams(max_tokens=m) for m in MAX_TOKENS]
    return [o.output_token_ids for o in LLM(_cfg("cuda"), model).generate(PROMPTS, params)]


def test_greedy_spec_matches_plain(model):
    ref = _plain(model)
    llm = LLM(_cfg("cuda", k=3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, [SamplingParams(max_tokens=m) for m in MAX_TOKENS])]
    assert got == ref
    assert llm.engine.runner.spec.stats["proposed"] > 0
    assert llm.engine.runner.spec_graphs, "uniform verify steps replay a captured graph"


def test_planted_drafts_all_accepted(model, monkeypatch):
    ref = _plain(model)
    by_prompt = {tuple(p): r for p, r in zip(PROMPTS, ref)}

    def oracle(self, out, hidden, accepted):
        for s in out.reqs:
            req = s.req
            if req.status.finished or req.num_computed_tokens != req.num_tokens - 1:
                continue
            n = len(req.output_token_ids)
            req.draft_token_ids = by_prompt[tuple(req.prompt_token_ids)][n:n + min(self.k, req.params.max_tokens - n - 1)]

    monkeypatch.setattr(spec_decode.SpecDecoder, "propose", oracle)
    llm = LLM(_cfg("cuda", k=3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, [SamplingParams(max_tokens=m) for m in MAX_TOKENS])]
    assert got == ref
    st = llm.engine.runner.spec.stats
    assert st["accepted"] == st["proposed"] > 0


def test_sampled_spec(model):
    llm = LLM(_cfg("cuda", k=3), model)
    got = llm.generate(PROMPTS, [SamplingParams(max_tokens=m, temperature=0.7) for m in MAX_TOKENS])
    assert [len(o.output_token_ids) for o in got] == MAX_TOKENS


def _hybrid_cfg(k=0, eager=False):
    from vllm_cmp170hx_b200.config import tiny

    m = tiny(layers=4, experts=8, layer_types=["kda", "mla", "kda", "kda"])
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                           max_model_len=512, num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=40), device="cuda", enforce_eager=eager,
                        cuda_graph_batch_sizes=[1, 2, 4])


@pytest.mark.parametrize("planted", [False, True])
def test_hybrid_kda_spec_matches_plain(planted, monkeypatch):
    """Verify steps through the KDA kernel record (u, k, decay) per token; the recover kernel applies
    the accepted prefix: greedy speculative output equals plain decoding on the GPU."""
    pstate.set_state(pstate.ParallelState())
    m = HybridForCausalLM(_hybrid_cfg().model, "cuda", seed=12)
    params = [SamplingParams(max_tokens=n) for n in MAX_TOKENS]
    ref = [o.output_token_ids for o in LLM(_hybrid_cfg(), m).generate(PROMPTS, params)]
    if planted:
        by_prompt = {tuple(p): r for p, r in zip(PROMPTS, ref)}

        def oracle(self, out, hidden, accepted):
            for s in out.reqs:
                req = s.req
                if req.status.finished or req.num_computed_tokens != req.num_tokens - 1:
                    continue
                n = len(req.output_token_ids)
                d = list(by_prompt[tuple(req.prompt_token_ids)][n:n + self.k])
                d = [t if i != 1 else (t + 1) % 500 for i, t in enumerate(d)]  # reject the second draft
                req.draft_token_ids = d[:max(0, min(self.k, req.params.max_tokens - n - 1))]

        monkeypatch.setattr(spec_decode.SpecDecoder, "propose", oracle)
    llm = LLM(_hybrid_cfg(k=3), m)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, params)]
    assert got == ref
    assert llm.engine.runner.spec_graphs, "uniform verify steps replay a captured graph"
    eager = LLM(_hybrid_cfg(k=3, eager=True), m)
    assert [o.output_token_ids for o in eager.generate(PROMPTS, params)] == ref
