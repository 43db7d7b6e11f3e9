"""Dev A/B switches and hot swaps flip implementations between steps; greedy outputs agree."""

import pytest

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.dev.ab import DevAB, HotSwap
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _cfg():
    return EngineConfig(model=tiny(layers=2, experts=4, expert_format="bf16"),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256),
                        cache=CacheConfig(num_blocks=24), device="cpu", enforce_eager=True)


def test_switch_flip_and_hot_swap():
    pstate.set_state(pstate.ParallelState())
    m = HybridForCausalLM(_cfg().model, "cpu", seed=4)
    prompts = [list(range(3, 30)), list(range(40, 52))]
    ref = [o.output_token_ids for o in LLM(_cfg(), m).generate(prompts, SamplingParams(max_tokens=4))]
    llm = LLM(_cfg(), m)
    ab = DevAB(llm.engine, "attention_splits")
    assert ab.flip() == "b" and ab.flip() == "a"
    with pytest.raises(KeyError):
        DevAB(llm.engine, "nope")
    hs = HotSwap(["gemm:torch"])
    hs.swap_in()
    try:
        got = [o.output_token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=4))]
    finally:
        hs.swap_out()
    assert got == ref


@pytest.mark.parametrize("name", ["async_scheduling", "shared_expert_stream", "kda_prefill", "exl3_tile_rows",
                                  "gemm_splitk", "prefix_caching", "fair_prefill", "router_dtype"])
def test_every_switch_flips_between_steps(name):
    """Generation flips the switch every step; both arms leave greedy outputs as they are (the switches
    whose arms change numerics are checked to reach their knob instead)."""
    from vllm_cmp170hx_b200 import envs

    pstate.set_state(pstate.ParallelState())
    m = HybridForCausalLM(_cfg().model, "cpu", seed=4)
    prompts = [list(range(3, 30)), list(range(40, 52))]
    ref = [o.output_token_ids for o in LLM(_cfg(), m).generate(prompts, SamplingParams(max_tokens=5))]
    import os

    names = ("VLLM_B200_SHARED_EXPERT_STREAM", "VLLM_B200_KDA_PREFILL", "VLLM_B200_EXL3_TILE_ROWS",
             "VLLM_B200_GEMM_SPLITK")
    saved = {v: os.environ.get(v) for v in names}  # the switch arms set them; put them back afterwards
    try:
        _flip_run(name, m, prompts, ref)
    finally:
        for v, val in saved.items():
            if val is None:
                os.environ.pop(v, None)
            else:
                os.environ[v] = val
        envs.reset_cache()


def _flip_run(name, m, prompts, ref):
    from vllm_cmp170hx_b200.dev.ab import SWITCHES

    llm = LLM(_cfg(), m)
    eng = llm.engine
    ab = DevAB(eng, name)
    for rid, p in zip("ab", prompts):
        eng.add_request(p, SamplingParams(max_tokens=5), rid)
    outs, flips = {}, 0
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o.output_token_ids
        ab.flip()
        flips += 1
    assert flips >= 5 and SWITCHES[name].doc
    if name == "router_dtype":
        assert all(layer.router_out is not None for layer in m.modules() if hasattr(layer, "router_out"))
    else:
        assert [outs["a"], outs["b"]] == ref
