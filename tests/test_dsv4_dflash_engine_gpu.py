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


def test_dsv4_model_generates_on_gpu_graph_equals_eager():
    """Decode steps of the DeepSeek-V4.1 layers run from CUDA graphs (the indexer's score width is a
    host bound, so no step reads the device) and emit the eager path's tokens."""
    pstate.set_state(pstate.ParallelState())
    m = tiny_dsv4(layers=3)

    def cfg(eager):
        return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                               max_model_len=512),
                            cache=CacheConfig(num_blocks=40), device="cuda", enforce_eager=eager)

    model = HybridForCausalLM(m, "cuda", seed=5)
    eager = LLM(cfg(True), model).generate(PROMPTS, SamplingParams(max_tokens=6))
    llm = LLM(cfg(False), model)
    graph = llm.generate(PROMPTS, SamplingParams(max_tokens=6))
    torch.cuda.synchronize()
    assert all(len(o.output_token_ids) == 6 for o in graph)
    assert all(0 <= t < m.vocab_size for o in graph for t in o.output_token_ids)
    assert llm.engine.runner.graphs, "no decode graph was captured"
    assert [o.output_token_ids for o in graph] == [o.output_token_ids for o in eager]
    llm.engine.runner.release_graphs()


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
