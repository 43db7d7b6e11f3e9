"""DeepSeek-V4.1 layers in the engine on CPU: generation does not depend on how prompts are chunked
(window rings, step scratch and paged groups), and greedy MTP speculative decoding (rejected
positions written and later overwritten, the ratio-2 carry ring) emits exactly the plain tokens."""

import pytest

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_dsv4
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate

PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]


def _cfg(budget, k=0):
    m = tiny_dsv4(layers=3)
    m.num_mtp_layers = 1 if k else 0
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=budget,
                                                           max_model_len=256, num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg(32).model, "cpu", seed=5)


def _gen(model, cfg, n=8):
    return [o.output_token_ids for o in LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=n))]


def test_generation_independent_of_chunking(model):
    a = _gen(model, _cfg(16))
    b = _gen(model, _cfg(128))
    assert a == b


def test_greedy_mtp_spec_matches_plain(model):
    plain = _gen(model, _cfg(64))
    llm = LLM(_cfg(64, k=3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, SamplingParams(max_tokens=8))]
    assert got == plain
    assert llm.engine.runner.spec.stats["proposed"] > 0
