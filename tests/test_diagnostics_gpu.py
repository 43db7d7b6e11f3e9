"""Light timing on the GPU: %globaltimer stamps recorded inside CUDA-graph replays land in the
row each replay opens (no host work per step)."""

import json

import numpy as np
import pytest

from vllm_cmp170hx_b200 import envs
from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.parallel import state as pstate
from vllm_cmp170hx_b200.utils import light_timing

pytestmark = pytest.mark.gpu


def test_light_timing_in_cuda_graphs(tmp_path, monkeypatch):
    pstate.set_state(pstate.ParallelState())
    envs.reset_cache()
    monkeypatch.setenv("VLLM_B200_LIGHT_TIMING", json.dumps({"rows": 64, "scopes": "layer", "dir": str(tmp_path)}))
    cfg = EngineConfig(model=tiny(layers=4, experts=8), scheduler=SchedulerConfig(max_num_seqs=4, max_model_len=512),
                       cache=CacheConfig(num_blocks=32), device="cuda", cuda_graph_batch_sizes=[1, 2, 4])
    eng = LLMEngine(cfg)
    for i in range(2):
        eng.add_request(list(range(3 + i, 40 + i)), SamplingParams(max_tokens=8))
    while eng.has_unfinished():
        eng.step()
    assert eng.runner.graphs  # decode ran as graph replays
    path = eng.runner.timer.dump()
    ring = np.load(path)["ring"]
    steps = ring[ring[:, 0] > 0][:, 0]
    assert len(steps) >= 8 and len(set(steps.tolist())) == len(steps)
    summ = light_timing.summarize(path)
    assert set(summ) == {"L0", "L1", "L2", "L3"} and all(0 < v < 1e5 for v in summ.values())
    envs.reset_cache()


def test_captured_gpu_calls_replay_on_the_oracle(tmp_path, monkeypatch):
    """Kernel calls saved from an eager GPU step replay on the CPU oracle within bf16 tolerance."""
    from vllm_cmp170hx_b200.utils import capture

    pstate.set_state(pstate.ParallelState())
    envs.reset_cache()
    spec = tmp_path / "cap.toml"
    spec.write_text(f'dir = "{tmp_path / "caps"}"\nops = ["gemm", "rms_norm"]\nmax_calls = 3\n')
    monkeypatch.setenv("VLLM_B200_CAPTURE", str(spec))
    cfg = EngineConfig(model=tiny(layers=4, experts=8), scheduler=SchedulerConfig(max_num_seqs=4, max_model_len=512),
                       cache=CacheConfig(num_blocks=32), device="cuda", enforce_eager=True)
    eng = LLMEngine(cfg)
    try:
        eng.add_request(list(range(5, 60)), SamplingParams(max_tokens=2))
        while eng.has_unfinished():
            eng.step()
    finally:
        eng.capture.uninstall()
        envs.reset_cache()
    d = tmp_path / "caps" / "rank0"
    lines = [json.loads(x) for x in (d / "index.jsonl").read_text().splitlines()]
    assert {x["op"] for x in lines} == {"gemm", "rms_norm"}
    for x in lines:
        rel = capture.replay(str(d / x["file"]), "cpu")
        assert rel < 2e-2, (x, rel)
