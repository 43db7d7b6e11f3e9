"""Engram memory on the GPU: the gate kernel against its fp32 definition, and the DeepSeek-V4.1-style
model with an Engram layer in the engine (logits against the CPU oracle path, CUDA-graph decode equal to
eager decode)."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_dsv4
from vllm_cmp170hx_b200.engine.llm_engine import LLM, LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.engram import gate_ref
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H", [(1, 256), (37, 2304), (300, 4096)])
def test_gate_kernel_matches_definition(T, H):
    g = torch.Generator().manual_seed(T + H)
    a = torch.randn(T, H, generator=g).bfloat16()
    h = torch.randn(T, H, generator=g).bfloat16()
    kv = torch.randn(T, 2 * H, generator=g).bfloat16()
    wh = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    wk = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    ref = gate_ref(a, h, kv, wh, wk, 1e-6).float()
    out = a.cuda()
    _ext.ops().engram_gate(h.cuda(), kv.cuda(), wh.cuda(), wk.cuda(), 1e-6, out)
    torch.cuda.synchronize()
    assert (out.cpu().float() - ref).abs().max() < 3e-2


def _cfg(device, eager=True):
    return EngineConfig(model=tiny_dsv4(layers=3, engram=True),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=512, max_model_len=512),
                        cache=CacheConfig(num_blocks=32), device=device, enforce_eager=eager,
                        cuda_graph_batch_sizes=[1, 2, 4])


def test_engram_model_matches_cpu_and_graphs_match_eager():
    pstate.set_state(pstate.ParallelState())
    prompts = [list(range(3, 3 + 90)), [5, 9, 11]]
    hs = {}
    for dev in ("cpu", "cuda"):
        model = HybridForCausalLM(_cfg(dev).model, dev, seed=3, init_mode="sliced")
        eng = LLMEngine(_cfg(dev), model)
        for p in prompts:
            eng.add_request(p, SamplingParams(max_tokens=1))
        out = eng.scheduler.schedule()
        h = eng.runner._host_inputs(out)
        d, ctx, _ = eng.runner._context(h)
        with torch.inference_mode():
            hidden = eng.runner.model(d["ids"], ctx)
            hs[dev] = eng.runner.model.compute_logits(hidden).float().cpu()
    rel = ((hs["cuda"] - hs["cpu"]).norm() / hs["cpu"].norm()).item()
    print(f"engram model logits rel {rel:.2e}")
    assert rel < 5e-2, rel
    p = SamplingParams(max_tokens=6)
    long_prompts = [list(range(10, 10 + n)) for n in (7, 66, 130)]
    eager = [o.output_token_ids for o in LLM(_cfg("cuda", eager=True), model).generate(long_prompts, p)]
    graph = [o.output_token_ids for o in LLM(_cfg("cuda", eager=False), model).generate(long_prompts, p)]
    assert eager == graph
