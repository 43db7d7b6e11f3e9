"""Sharded checkpoints: a saved model reloads into a freshly built one (different random init) and
generates the same tokens; layout and shape mismatches are refused."""

import pytest

from vllm_cmp170hx_b200 import checkpoint
from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny, tiny_deepseek
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


@pytest.mark.parametrize("which", ["exl3", "deepseek"])
def test_save_load_roundtrip(tmp_path, which):
    pstate.set_state(pstate.ParallelState())
    mcfg = tiny(layers=2, experts=4) if which == "exl3" else tiny_deepseek(layers=2, experts=4, vocab=512)
    cfg = EngineConfig(model=mcfg, scheduler=SchedulerConfig(max_num_seqs=2, max_model_len=256),
                       cache=CacheConfig(num_blocks=16), device="cpu", enforce_eager=True)
    a = HybridForCausalLM(mcfg, "cpu", seed=1)
    checkpoint.save(a, str(tmp_path))
    b = HybridForCausalLM(mcfg, "cpu", seed=2)
    prompts = [list(range(5, 25))]
    p = SamplingParams(max_tokens=3)
    before = LLM(cfg, b).generate(prompts, p)[0].output_token_ids
    checkpoint.load(b, str(tmp_path))
    assert LLM(cfg, b).generate(prompts, p)[0].output_token_ids == LLM(cfg, a).generate(prompts, p)[0].output_token_ids
    assert before is not None
    other = HybridForCausalLM(tiny(layers=3, experts=4), "cpu", seed=1)
    with pytest.raises(checkpoint.CheckpointMismatch):
        checkpoint.load(other, str(tmp_path))
