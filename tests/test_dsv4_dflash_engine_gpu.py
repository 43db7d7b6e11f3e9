"""The engine on the GPU with the newer pieces: a DeepSeek-V4.1-style model (window + compressed
sparse attention on the 512-wide sink attention kernel, delayed mHC, EXL3 experts) generating
eagerly, and DFlash speculative decoding on the hybrid model emitting exactly the plain greedy
tokens."""

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny, tiny_dsv4
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate

pytestmark = pytest.mark.gpu

PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71, 150])]


def test_dsv4_model_generates_on_gpu():
    pstate.set_state(pstate.ParallelState())
    m = tiny_dsv4(layers=3)
    cfg = EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=512),
                       cache=CacheConfig(num_blocks=40), device="cuda")
    model = HybridForCausalLM(m, "cuda", seed=5)
    outs = LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=6))
    torch.cuda.synchronize()
    assert all(len(o.output_token_ids) == 6 for o in outs)
    assert all(0 <= t < m.vocab_size for o in outs for t in o.output_token_ids)


def test_dflash_spec_matches_plain_on_gpu():
    pstate.set_state(pstate.ParallelState())
    m = tiny(layers=4, experts=8, hidden=256, expert_format="exl3")

    def cfg(k):
        return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                               max_model_len=512, num_speculative_tokens=k,
                                                               spec_method="dflash"),
                            cache=CacheConfig(num_blocks=40), device="cuda", enforce_eager=True)

    model = HybridForCausalLM(m, "cuda", seed=7)
    plain = [o.output_token_ids for o in LLM(cfg(0), model).generate(PROMPTS, SamplingParams(max_tokens=8))]
    llm = LLM(cfg(3), model)
    got = [o.output_token_ids for o in llm.generate(PROMPTS, SamplingParams(max_tokens=8))]
    model.aux_layer_ids = ()
    assert got == plain
    assert llm.engine.runner.spec.stats["proposed"] > 0
