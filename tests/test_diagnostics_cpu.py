"""Diagnostics on CPU: light timing (host-clock path), state index checks, kernel-call capture,
memory attribution / KV plan, serial trace export ordering, execution traces, env gates."""

import json
import os
import threading
import time

import numpy as np
import pytest
import torch

from vllm_cmp170hx_b200 import envs
from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.parallel import state as pstate
from vllm_cmp170hx_b200.utils import light_timing, memory, state_check, trace
from vllm_cmp170hx_b200.utils.capture import KernelCapture


def _cfg():
    return EngineConfig(model=tiny(layers=2, experts=4, expert_format="bf16"),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256),
                        cache=CacheConfig(num_blocks=24), device="cpu", enforce_eager=True)


@pytest.fixture(autouse=True)
def _state(monkeypatch):
    pstate.set_state(pstate.ParallelState())
    envs.reset_cache()
    yield
    envs.reset_cache()


def _run(eng, n=2, steps=100):
    for i in range(n):
        eng.add_request(list(range(5 + i, 20 + i)), SamplingParams(max_tokens=3))
    k = 0
    while eng.has_unfinished() and k < steps:
        eng.step()
        k += 1


def test_light_timing_rows_and_summary(tmp_path, monkeypatch):
    monkeypatch.setenv("VLLM_B200_LIGHT_TIMING", json.dumps({"rows": 16, "scopes": "block", "dir": str(tmp_path)}))
    eng = LLMEngine(_cfg())
    assert eng.runner.timer is not None
    _run(eng)
    path = eng.runner.timer.dump()
    d = np.load(path)
    assert (d["ring"][:, 0] > 0).sum() >= 3  # one row per forward
    summ = light_timing.summarize(path)
    assert {"L0", "L1", "L0.attn", "L0.mlp"} <= set(summ) and all(v >= 0 for v in summ.values())


def test_state_index_check_raises(monkeypatch):
    monkeypatch.setenv("VLLM_B200_STATE_INDEX_CHECK", "1")
    eng = LLMEngine(_cfg())
    eng.add_request(list(range(10)), SamplingParams(max_tokens=2))
    out = eng.scheduler.schedule()
    h = eng.runner._host_inputs(out)  # valid inputs pass
    h["slots"][0] = eng.runner.num_blocks * 64 + 5
    with pytest.raises(state_check.StateIndexError):
        state_check.check_step(h, out, eng.runner.num_blocks, 64, eng.runner.num_slots, 256)
    out.reqs[0].req.block_ids[0] = eng.runner.num_blocks + 3  # corrupt the block table
    with pytest.raises(state_check.StateIndexError, match="slot mapping|block table"):
        eng.runner._host_inputs(out)


def test_kernel_capture_writes_calls(tmp_path, monkeypatch):
    spec = tmp_path / "cap.toml"
    spec.write_text(f'dir = "{tmp_path / "caps"}"\nops = ["gemm", "rms_norm"]\nmax_calls = 2\n')
    monkeypatch.setenv("VLLM_B200_CAPTURE", str(spec))
    eng = LLMEngine(_cfg())
    try:
        _run(eng, n=1)
    finally:
        eng.capture.uninstall()
    d = tmp_path / "caps" / "rank0"
    lines = [json.loads(x) for x in (d / "index.jsonl").read_text().splitlines()]
    assert {x["op"] for x in lines} == {"gemm", "rms_norm"} and len(lines) == 4
    rec = torch.load(d / lines[0]["file"])
    assert isinstance(rec["out"], torch.Tensor) and rec["args"]
    # every saved call replays to its saved result (the CPU path is deterministic), also through the CLI
    from vllm_cmp170hx_b200.utils import capture

    assert all(capture.replay(str(d / x["file"])) == 0.0 for x in lines)
    assert capture.main(["replay", str(d), "--tol", "0"]) == 0
    # a corrupted result is reported
    rec["out"] = rec["out"] + 1
    torch.save(rec, d / lines[0]["file"])
    assert capture.replay(str(d / lines[0]["file"])) > 0
    assert capture.main(["replay", str(d), "--tol", "0"]) == 1


def test_memory_attribution_and_kv_plan():
    eng = LLMEngine(_cfg())
    a = memory.attribute(eng.runner.model)
    total = sum(p.numel() * p.element_size() for p in eng.runner.model.parameters())
    assert a["routed_experts"] > 0 and a["embedding"] > 0 and sum(a.values()) >= total
    plan = memory.kv_plan(eng.runner)
    assert plan["blocks"] == 24 and plan["tokens_capacity"] == 24 * 64


def test_serial_export_order(tmp_path):
    class FakeProf:
        def __init__(self, log, r):
            self.log, self.r = log, r

        def export_chrome_trace(self, p):
            self.log.append(self.r)
            open(p, "w").write("{}")

    log = []
    world = 4
    ths = [threading.Thread(target=trace.serial_export,
                            args=(FakeProf(log, r), str(tmp_path / f"r{r}.json"), r, world, str(tmp_path)))
           for r in reversed(range(world))]
    for t in ths:
        t.start()
        time.sleep(0.01)
    for t in ths:
        t.join(timeout=30)
    assert log == [0, 1, 2, 3]


def test_engine_profile_writes_trace(tmp_path, monkeypatch):
    monkeypatch.setenv("VLLM_B200_EXECUTION_TRACE", "1")
    eng = LLMEngine(_cfg())
    eng.add_request(list(range(12)), SamplingParams(max_tokens=4))
    path = eng.profile(2, str(tmp_path))
    assert os.path.exists(path) and os.path.exists(os.path.join(tmp_path, "rank0.et.json"))
