"""Verify width per step from the requests' last verified rounds (the depth hint table)."""

import os

import pytest

from vllm_cmp170hx_b200.engine.depth_hint import DepthHint, certain_output
from vllm_cmp170hx_b200.engine.request import Request, SamplingParams


def _req(rid, certain=False):
    return Request([1, 2, 3], SamplingParams(max_tokens=8, certain_output=certain), request_id=rid)


def test_parse_and_widths():
    h = DepthHint.parse("full=7,7,5,5;base=5,5,5,3")
    assert h.full == (7, 7, 5, 5) and h.base == (5, 5, 5, 3)
    assert [h.width("full", n) for n in (0, 1, 3, 4, 9)] == [7, 7, 5, 5, 5]  # the last entry repeats
    assert h.width("base", 12) == 3
    assert DepthHint.parse("") is None and DepthHint.parse("  ") is None
    for bad in ("full=7", "full=7;base=x", "full=7;base=5;deep=3", "full=;base=5"):
        with pytest.raises(ValueError):
            DepthHint.parse(bad)


def test_select_full_only_when_every_decoder_had_a_full_round():
    h = DepthHint.parse("full=6,6,4;base=3,3,2")
    a, b, c = _req("a"), _req("b"), _req("c", certain=True)
    assert h.select([a, b], 2, 8) == 3  # first decoding step: base
    h.observe("a", 3, 3)
    h.observe("b", 3, 1)
    assert h.select([a, b], 2, 8) == 3  # b's last round was not full
    h.observe("b", 3, 3)
    assert h.select([a, b], 2, 8) == 6
    assert h.select([a, b], 2, 5) == 5  # capped by the adaptive width
    assert h.select([a, b, c], 3, 8) == 4  # c is certain by its own fields; the load picks entry 3
    h.observe("a", 0, 0)  # a step without drafts says nothing
    assert h.rounds["a"] is True
    h.forget("a")
    assert h.select([a], 1, 8) == 3
    assert h.select([], 1, 8) == 3


def test_certain_output_from_chat_fields():
    assert certain_output({"tools": [{"type": "function"}]})
    assert not certain_output({"tools": [{"type": "function"}], "tool_choice": "none"})
    assert certain_output({"response_format": {"type": "json_schema"}})
    assert not certain_output({"response_format": {"type": "text"}})
    assert not certain_output({})


def test_engine_caps_verified_drafts_by_the_hint():
    """With full=2;base=1, the first verify steps check one draft, later ones two once every decoding
    request accepted all its drafts; greedy outputs equal those without the hint."""
    from vllm_cmp170hx_b200 import envs
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_deepseek
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    m = tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512)

    def cfg():
        return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                               max_model_len=256, num_speculative_tokens=3),
                            cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)

    model = HybridForCausalLM(m, "cpu", seed=5)
    prompts = [[(7 * i + j) % 500 for j in range(11 + 5 * i)] for i in range(2)]
    ref = [o.output_token_ids for o in LLM(cfg(), model).generate(prompts, SamplingParams(max_tokens=10))]
    saved = os.environ.get("VLLM_B200_DEPTH_HINT")
    os.environ["VLLM_B200_DEPTH_HINT"] = "full=2;base=1"
    envs.reset_cache()
    try:
        llm = LLM(cfg(), model)
        eng = llm.engine
        assert eng.depth_hint is not None
        caps = []
        orig = eng.scheduler.schedule

        def schedule(*a, **k):
            out = orig(*a, **k)
            caps.extend(s.num_draft for s in out.reqs if s.num_draft)
            return out

        eng.scheduler.schedule = schedule
        got = [o.output_token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10))]
    finally:
        if saved is None:
            os.environ.pop("VLLM_B200_DEPTH_HINT", None)
        else:
            os.environ["VLLM_B200_DEPTH_HINT"] = saved
        envs.reset_cache()
    assert got == ref
    assert caps and max(caps) <= 2 and caps[0] == 1
