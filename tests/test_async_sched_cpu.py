"""Asynchronous scheduling on CPU (eager launches, the same bookkeeping as the GPU's graph replays):
every request gets exactly the tokens of synchronous scheduling -- with stop tokens that end requests
while the next step is already launched, length limits, requests arriving between steps and an abort."""

import pytest

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _cfg(async_on):
    return EngineConfig(model=tiny(layers=4, experts=8, expert_format="bf16"),
                        scheduler=SchedulerConfig(max_num_seqs=6, max_num_batched_tokens=256, max_model_len=256,
                                                  async_scheduling=async_on),
                        cache=CacheConfig(num_blocks=40), device="cpu", enforce_eager=True,
                        cuda_graph_batch_sizes=[1, 2, 4, 8])


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg(False).model, "cpu", seed=21)


def _run(model, async_on, plan):
    """plan: {step number: [(request id, prompt, params)]}; request 'abort@k' ids abort at step k."""
    eng = LLMEngine(_cfg(async_on), model)
    outs, steps, aborted = {}, 0, False
    while steps < 200:
        for rid, prompt, params in plan.get(steps, []):
            eng.add_request(prompt, params, rid)
        if steps == 9 and not aborted:
            eng.abort_request("r2")
            aborted = True
        for o in eng.step():
            outs[o.request_id] = (o.output_token_ids, o.finish_reason)
        steps += 1
        if not eng.has_unfinished() and steps > max(plan):
            break
    return outs, eng


def test_async_matches_sync(model):
    # a stop token that greedy decoding emits for some requests, found from a synchronous run
    probe, _ = _run(model, False, {0: [("p", list(range(30, 60)), SamplingParams(max_tokens=12))]})
    stop = probe["p"][0][4]
    plan = {
        0: [("r0", list(range(10, 40)), SamplingParams(max_tokens=10)),
            ("r1", list(range(30, 60)), SamplingParams(max_tokens=12, stop_token_ids=[stop])),
            ("r2", list(range(5, 25)), SamplingParams(max_tokens=30))],
        3: [("r3", list(range(50, 70)), SamplingParams(max_tokens=6))],
        6: [("r4", list(range(1, 90)), SamplingParams(max_tokens=1)),
            ("r5", list(range(7, 17)), SamplingParams(max_tokens=8))],
    }
    sync, _ = _run(model, False, plan)
    asy, eng = _run(model, True, plan)
    assert asy["r1"][1] == "stopped" and len(asy["r1"][0]) == 5  # stopped while a step was in flight
    for rid in ("r0", "r1", "r3", "r4", "r5"):
        assert asy[rid] == sync[rid], rid
    assert asy["r2"][0] == sync["r2"][0][:len(asy["r2"][0])]
    assert not eng.scheduler.running and not eng.requests
