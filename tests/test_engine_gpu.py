"""The engine on the GPU: the tiny hybrid model's logits vs the same model on
the CPU oracle path, and CUDA-graph decode vs eager decode."""

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLM, LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.engine.scheduler import ScheduledReq, SchedulerOutput
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate

pytestmark = pytest.mark.gpu


def _cfg(device, eager=True, fmt="exl3"):
    return EngineConfig(model=tiny(layers=4, experts=8, expert_format=fmt),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=512, max_model_len=512),
                        cache=CacheConfig(num_blocks=32), device=device, enforce_eager=eager,
                        cuda_graph_batch_sizes=[1, 2, 4])


@pytest.mark.parametrize("fmt", ["exl3", "bf16"])
def test_gpu_forward_matches_cpu_oracle(fmt):
    pstate.set_state(pstate.ParallelState())
    prompts = [list(range(3, 3 + 90)), [5, 9, 11]]
    hs = {}
    for dev in ("cpu", "cuda"):
        model = HybridForCausalLM(_cfg(dev, fmt=fmt).model, dev, seed=3, init_mode="sliced")
        eng = LLMEngine(_cfg(dev, fmt=fmt), model)
        for p in prompts:
            eng.add_request(p, SamplingParams(max_tokens=1))
        out = eng.scheduler.schedule()
        h = eng.runner._host_inputs(out)
        d, ctx, _ = eng.runner._context(h)
        with torch.inference_mode():
            hidden = eng.runner.model(d["ids"], ctx)
            hs[dev] = eng.runner.model.compute_logits(hidden).float().cpu()
    rel = ((hs["cuda"] - hs["cpu"]).norm() / hs["cpu"].norm()).item()
    assert rel < 5e-2, rel


def test_graph_decode_matches_eager():
    pstate.set_state(pstate.ParallelState())
    model = HybridForCausalLM(_cfg("cuda").model, "cuda", seed=4, init_mode="local")
    prompts = [list(range(10, 10 + n)) for n in (7, 66, 130)]
    p = SamplingParams(max_tokens=6)
    eager = LLM(_cfg("cuda", eager=True), model).generate(prompts, p)
    graph = LLM(_cfg("cuda", eager=False), model).generate(prompts, p)
    for a, b in zip(eager, graph):
        assert a.output_token_ids == b.output_token_ids


def test_banned_tokens_in_kernel_and_graph():
    """The sampling kernel skips each row's banned ids (against the CPU reference of the same rule), and
    a graph-captured decode step applies them from its input buffer."""
    from vllm_cmp170hx_b200.ops import sampling as sampling_ops

    g = torch.Generator(device="cuda").manual_seed(0)
    logits = torch.randn(6, 1000, device="cuda", generator=g).bfloat16()
    top = logits.float().argmax(-1)
    bans = torch.full((6, 4), -1, dtype=torch.int32, device="cuda")
    bans[:, 0] = top.int()
    bans[1, 1] = logits[1].float().topk(2).indices[1].int()
    for off in (0, 500):  # the vocab shard's offset
        shard_bans = torch.where(bans >= 0, bans + off, bans).int().contiguous()
        val, idx = sampling_ops.sample_local(logits, None, 0, None, off, shard_bans)
        v_ref, i_ref = sampling_ops.sample_local(logits.cpu(), None, 0, None, off, shard_bans.cpu())
        assert idx.cpu().tolist() == i_ref.tolist()
        assert all(int(i) - off != int(t) for i, t in zip(idx.cpu(), top.cpu()))
    pstate.set_state(pstate.ParallelState())
    model = HybridForCausalLM(_cfg("cuda").model, "cuda", seed=4, init_mode="local")
    prompts = [list(range(10, 10 + n)) for n in (7, 66)]
    free = LLM(_cfg("cuda", eager=False), model).generate(prompts, SamplingParams(max_tokens=4))
    ban = free[0].output_token_ids[2]
    ps = [SamplingParams(max_tokens=4, bad_token_ids=[ban]), SamplingParams(max_tokens=4)]
    for eager in (True, False):
        out = LLM(_cfg("cuda", eager=eager), model).generate(prompts, ps)
        assert ban not in out[0].output_token_ids
        assert out[1].output_token_ids == free[1].output_token_ids


def test_kv_pool_sized_from_a_profiled_step():
    """With num_blocks = 0 the runner measures one full prefill step's activation peak and sizes the KV
    pool from the free memory left: the peak is positive, the pool covers every sequence, and the
    engine generates with it."""
    pstate.set_state(pstate.ParallelState())
    cfg = EngineConfig(model=tiny(layers=4, experts=8), device="cuda", enforce_eager=False,
                       scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=512, max_model_len=512),
                       cache=CacheConfig(num_blocks=0, gpu_memory_utilization=0.5), cuda_graph_batch_sizes=[1, 2, 4])
    model = HybridForCausalLM(cfg.model, "cuda", seed=4, init_mode="local")
    llm = LLM(cfg, model)
    r = llm.engine.runner
    assert r.activation_peak > 0
    assert r.num_blocks == cfg.scheduler.max_num_seqs * r.max_blocks_per_seq + 1
    outs = llm.generate([list(range(10, 10 + n)) for n in (7, 130)], SamplingParams(max_tokens=4))
    assert all(len(o.output_token_ids) == 4 for o in outs)


def test_shared_expert_stream_matches_inline(monkeypatch):
    """With the shared expert on a second stream (fork / join, also inside the decode graphs) the engine
    emits the tokens of the inline order; graph capture reports kept and transient bytes."""
    from vllm_cmp170hx_b200 import envs

    pstate.set_state(pstate.ParallelState())
    model = HybridForCausalLM(_cfg("cuda").model, "cuda", seed=6, init_mode="local")
    prompts = [list(range(20, 20 + n)) for n in (5, 70, 129)]
    p = SamplingParams(max_tokens=5)
    base = [o.output_token_ids for o in LLM(_cfg("cuda", eager=False), model).generate(prompts, p)]
    envs.reset_cache()
    monkeypatch.setenv("VLLM_B200_SHARED_EXPERT_STREAM", "1")
    try:
        for eager in (True, False):
            llm = LLM(_cfg("cuda", eager=eager), model)
            assert [o.output_token_ids for o in llm.generate(prompts, p)] == base
        eng = LLMEngine(_cfg("cuda", eager=False), model)
        kept = eng.warmup()
        assert set(kept) == {1, 2, 4} and all(v >= 0 for v in kept.values())
        assert set(eng.runner.graph_transient) == {1, 2, 4}
    finally:
        envs.reset_cache()


def test_async_scheduling_matches_sync():
    """Decode steps scheduled and launched one step ahead (input ids gathered on the device from the
    previous graph's sampled tokens) emit the synchronous tokens, also when a stop token ends a request
    while the next step is in flight and when requests arrive mid-run."""
    pstate.set_state(pstate.ParallelState())
    model = HybridForCausalLM(_cfg("cuda").model, "cuda", seed=8, init_mode="local")

    def run(async_on, stop=None):
        cfg = _cfg("cuda", eager=False)
        cfg.scheduler.async_scheduling = async_on
        eng = LLMEngine(cfg, model)
        outs = {}
        plan = {0: [("a", list(range(10, 50)), 12), ("b", list(range(60, 75)), 9)], 4: [("c", [3, 4, 5], 7)]}
        for step in range(100):
            for rid, prompt, n in plan.get(step, []):
                eng.add_request(prompt, SamplingParams(max_tokens=n, stop_token_ids=[stop] if stop else []), rid)
            for o in eng.step():
                outs[o.request_id] = (o.output_token_ids, o.finish_reason)
            if step > 4 and not eng.has_unfinished():
                break
        return outs

    sync = run(False)
    assert run(True) == sync
    stop = sync["a"][0][5]
    assert run(True, stop) == run(False, stop)
