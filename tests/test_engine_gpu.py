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
