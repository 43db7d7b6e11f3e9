"""End-to-end engine on CPU (oracle path): tiny hybrid model, chunked prefill,
continuous batching, greedy determinism, chunking invariance."""

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLM, LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _cfg(max_tokens_per_step=64, layer_types=None, expert_format="bf16"):
    m = tiny(layers=4, experts=4, expert_format=expert_format, layer_types=layer_types)
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=max_tokens_per_step,
                                                           max_model_len=512),
                        cache=CacheConfig(num_blocks=64), device="cpu", enforce_eager=True)


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    torch.manual_seed(0)
    return HybridForCausalLM(_cfg().model, "cpu", seed=1, init_mode="sliced")


def test_generate_and_chunking_invariance(model):
    prompts = [[(7 * i + j) % 500 for j in range(n)] for i, n in enumerate([5, 37, 70])]
    p = SamplingParams(max_tokens=4)
    a = LLM(_cfg(max_tokens_per_step=256), model).generate(prompts, p)
    b = LLM(_cfg(max_tokens_per_step=16), model).generate(prompts, p)  # prompts chunked
    for x, y in zip(a, b):
        assert len(x.output_token_ids) == 4
        assert x.output_token_ids == y.output_token_ids


def test_batching_invariance(model):
    prompts = [[(3 * i + 11 * j) % 500 for j in range(20 + i)] for i in range(3)]
    p = SamplingParams(max_tokens=3)
    together = LLM(_cfg(), model).generate(prompts, p)
    alone = [LLM(_cfg(), model).generate([pr], p)[0] for pr in prompts]
    for x, y in zip(together, alone):
        assert x.output_token_ids == y.output_token_ids


def test_engine_step_outputs(model):
    eng = LLMEngine(_cfg(), model)
    rid = eng.add_request(list(range(10)), SamplingParams(max_tokens=2))
    outs = []
    while eng.has_unfinished():
        outs += eng.step()
    fin = [o for o in outs if o.finished]
    assert len(fin) == 1 and fin[0].request_id == rid and fin[0].finish_reason == "length"


def test_failed_input_isolation():
    """A request whose prompt contains a token with a NaN embedding finishes with an error; the
    other requests in the batch finish normally with the tokens they produce alone."""
    pstate.set_state(pstate.ParallelState())
    m = HybridForCausalLM(_cfg().model, "cpu", seed=2, init_mode="sliced")
    good = [[(5 * j + 1) % 400 for j in range(20)], [(7 * j + 3) % 400 for j in range(33)]]
    alone = [o.output_token_ids for o in LLM(_cfg(), m).generate(good, SamplingParams(max_tokens=4))]
    m.embed.data[450] = float("nan")
    bad = [11, 12, 450, 13]
    outs = LLM(_cfg(), m).generate([good[0], bad, good[1]], SamplingParams(max_tokens=4))
    assert outs[1].finish_reason == "error" and outs[1].output_token_ids == []
    assert [outs[0].output_token_ids, outs[2].output_token_ids] == alone


def test_warmup_leaves_pools_free(model):
    eng = LLMEngine(_cfg(), model)
    free = eng.runner.block_pool.num_free()
    eng.warmup()
    assert eng.runner.block_pool.num_free() == free
    out = eng.step()  # nothing scheduled
    assert out == [] and not eng.has_unfinished()


def test_decode_step_inputs_fast_path_equals_general_path():
    """The vectorised decode-step input builder gives the general builder's arrays (with padding)."""
    import numpy as np

    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = EngineConfig(model=tiny(layers=2, experts=4, hidden=256),
                       scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=512, max_model_len=512),
                       cache=CacheConfig(num_blocks=64), device="cpu", enforce_eager=True)
    eng = LLMEngine(cfg, HybridForCausalLM(cfg.model, "cpu", seed=0))
    for i, n in enumerate([5, 70, 130]):
        eng.add_request([(3 * i + j) % 400 + 1 for j in range(n)],
                        SamplingParams(max_tokens=20, temperature=0.5 * (i % 2)))
    for _ in range(3):
        eng.step()
    out = eng.scheduler.schedule()
    r = eng.runner
    assert out.decode_only and all(s.num_new == 1 for s in out.reqs)
    for pad in (None, 8):
        fast = r._host_inputs(out, pad_to=pad)
        r._check_indices = True  # forces the general builder
        try:
            gen = r._host_inputs(out, pad_to=pad)
        finally:
            r._check_indices = False
        for k in ("ids", "pos", "slots", "tseq", "ctx", "cu", "kslot", "hinit", "bt", "temps", "sample_rows"):
            assert np.array_equal(fast[k], gen[k]), (pad, k, fast[k], gen[k])
        assert (fast["max_ctx"], fast["T"], fast["S"]) == (gen["max_ctx"], gen["T"], gen["S"])


def test_synthetic_prefix_skips_prefill(model):
    """A request with a synthetic prefix starts at that position: its first step computes the last
    prompt token only, over the rows the caches hold (here filled with random values)."""
    eng = LLMEngine(_cfg(max_tokens_per_step=256), model)
    eng.runner.fill_caches_random(3)
    ids = [eng.add_request([(5 * j) % 500 for j in range(100)], SamplingParams(max_tokens=3), synthetic_prefix=99)
           for _ in range(2)]
    out = eng.scheduler.schedule()
    assert [s.num_new for s in out.reqs] == [1, 1] and all(s.start == 99 and s.sample for s in out.reqs)
    eng.scheduler.waiting.extendleft(reversed([s.req for s in out.reqs]))  # undo: let step() schedule them
    for s in out.reqs:
        eng.scheduler.running.remove(s.req)
        eng.scheduler._release(s.req)
        s.req.num_computed_tokens = 0
    done = {}
    while eng.has_unfinished():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o
    assert sorted(done) == sorted(ids) and all(len(o.output_token_ids) == 3 for o in done.values())


def _mla_cfg(prefix_caching):
    from vllm_cmp170hx_b200.config import tiny_deepseek

    m = tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512)
    m.mla.attn_weight_format = "bf16"
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=512,
                                                           max_model_len=512),
                        cache=CacheConfig(num_blocks=32, enable_prefix_caching=prefix_caching), device="cpu",
                        enforce_eager=True)


def test_prefix_caching_reuses_blocks_and_keeps_outputs():
    """A second request sharing a 2-block prefix with a finished one starts after the cached blocks and
    generates what it generates without the cache."""
    pstate.set_state(pstate.ParallelState())
    base = [(13 * j) % 500 for j in range(150)]
    prompts = [base + [1, 2, 3], base[:140] + [7, 8]]
    p = SamplingParams(max_tokens=3)
    model = HybridForCausalLM(_mla_cfg(False).model, "cpu", seed=2, init_mode="sliced")
    ref = [o.output_token_ids for o in LLM(_mla_cfg(False), model).generate(prompts, p)]
    eng = LLMEngine(_mla_cfg(True), model)
    outs = []
    for prompt in prompts:  # one after the other: the second sees the first's registered blocks
        eng.add_request(prompt, p)
        while eng.has_unfinished():
            for o in eng.step():
                if o.finished:
                    outs.append(o.output_token_ids)
    assert outs == ref
    assert eng.scheduler.prefix_hits == 128  # two full 64-token blocks of the shared prefix


def test_banned_tokens_are_never_sampled(model):
    """A request's bad_token_ids (the decode mask of a tool_choice="none" request) never win: with the
    greedy tokens of a first run banned, every step picks another token."""
    prompts = [[(5 * i + 3 * j) % 500 for j in range(12 + 5 * i)] for i in range(3)]
    free = LLM(_cfg(), model).generate(prompts, SamplingParams(max_tokens=1))
    firsts = [o.output_token_ids[0] for o in free]
    banned = [LLM(_cfg(), model).generate([p], SamplingParams(max_tokens=4, bad_token_ids=[t]))[0]
              for p, t in zip(prompts, firsts)]
    for o, t in zip(banned, firsts):
        assert t not in o.output_token_ids
    # the other requests of a batch are not affected
    mixed = LLM(_cfg(), model).generate(prompts, [SamplingParams(max_tokens=1, bad_token_ids=[firsts[0]]),
                                                  SamplingParams(max_tokens=1), SamplingParams(max_tokens=1)])
    assert mixed[0].output_token_ids[0] != firsts[0]
    assert [o.output_token_ids[0] for o in mixed[1:]] == firsts[1:]
