"""Every declared VLLM_B200_* flag is read by the code path it names, and the reference's names of
behaviours that are always on here are reported as such (one test per flag family)."""

import os
import re

import pytest

from vllm_cmp170hx_b200 import envs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "vllm_cmp170hx_b200")


def _sources():
    for d, _, files in os.walk(PKG):
        for f in files:
            if f.endswith((".py", ".cu", ".cpp", ".h", ".cuh")) and f != "envs.py":
                with open(os.path.join(d, f)) as h:
                    yield h.read()


def test_every_declared_flag_is_read_somewhere():
    text = "\n".join(_sources())
    dead = [n for n in envs.VARS if not re.search(re.escape(f'"{n}"'), text)]
    assert not dead, dead


@pytest.fixture
def env(monkeypatch):
    envs.reset_cache()
    yield monkeypatch
    envs.reset_cache()


def test_tile_rows_and_splits_flags(env):
    from vllm_cmp170hx_b200.ops.mla import pick_splits
    from vllm_cmp170hx_b200.ops.moe import pick_tile_rows

    assert pick_tile_rows(128, 8, 256) == 16
    env.setenv("VLLM_B200_EXL3_TILE_ROWS", "64")
    envs.reset_cache()
    assert pick_tile_rows(128, 8, 256) == 64
    env.setenv("VLLM_B200_SPARSE_MLA_SPLITS", "3")
    envs.reset_cache()
    assert pick_splits(64, 128) == 3


def test_short_prompt_bypass_flag(env):
    from vllm_cmp170hx_b200.config import CacheConfig, SchedulerConfig
    from vllm_cmp170hx_b200.engine.block_pool import make_block_pool
    from vllm_cmp170hx_b200.engine.request import Request, SamplingParams
    from vllm_cmp170hx_b200.engine.scheduler import Scheduler

    def admitted():
        s = Scheduler(SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=80, max_model_len=512,
                                      max_num_partial_prefills=1, long_prefill_token_threshold=64),
                      CacheConfig(num_blocks=64), make_block_pool(64, 1))
        s.add(Request(list(range(200)), SamplingParams(max_tokens=2)))  # long: partial prefill
        s.add(Request(list(range(20)), SamplingParams(max_tokens=2)))
        return [r.num_new for r in s.schedule().reqs]

    assert admitted() == [64]  # the short prompt does not fit the 16 tokens left: it waits
    env.setenv("VLLM_B200_FAIR_PREFILL_SHORT_BYPASS", "32")
    envs.reset_cache()
    assert admitted() == [64, 16]  # a short prompt is not held back by the partial-prefill cap


def test_cuda_graphs_flag_forces_eager(env):
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    env.setenv("VLLM_B200_CUDA_GRAPHS", "0")
    envs.reset_cache()
    cfg = EngineConfig(model=tiny(layers=2, experts=4), scheduler=SchedulerConfig(max_num_seqs=2, max_model_len=128),
                       cache=CacheConfig(num_blocks=8), device="cpu")
    LLMEngine(cfg)
    assert cfg.enforce_eager


def test_always_on_reference_names_are_reported(env):
    env.setenv("VLLM_PP_PACKED_HOP", "1")
    msgs = envs.check_environment()
    assert any("VLLM_PP_PACKED_HOP has no effect here" in m for m in msgs)


def test_transport_flags_are_validated(env):
    env.setenv("VLLM_B200_EP_DISPATCH", "bogus")
    envs.reset_cache()
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = EngineConfig(model=tiny(layers=2, experts=4), scheduler=SchedulerConfig(max_num_seqs=2, max_model_len=128),
                       cache=CacheConfig(num_blocks=8), device="cpu")
    with pytest.raises(ValueError, match="VLLM_B200_EP_DISPATCH"):
        LLMEngine(cfg)


def test_tuning_table_drives_the_cut_offs(env, tmp_path):
    """A card table given by VLLM_B200_TUNING_FILE replaces the cut-offs the kernels' launchers use."""
    from vllm_cmp170hx_b200 import tuning_table
    from vllm_cmp170hx_b200.ops.mla import pick_splits
    from vllm_cmp170hx_b200.ops.moe import pick_tile_rows

    table = tmp_path / "card.toml"
    table.write_text('schema = "b200-tuning/1"\ncard = "test"\n'
                     '[[row]]\nop = "exl3_moe"\nparam = "tile_rows_by_avg_rows"\nkey = {}\n'
                     'value = [[100, 64]]\nevidence = "test"\n'
                     '[[row]]\nop = "sparse_mla"\nparam = "max_splits"\nkey = {}\nvalue = 1\nevidence = "test"\n')
    env.setenv("VLLM_B200_TUNING_FILE", str(table))
    envs.reset_cache()
    tuning_table._table.cache_clear()
    tuning_table._lookup.cache_clear()
    try:
        assert pick_tile_rows(128, 8, 256) == 64
        assert pick_splits(1, 16, 2048) == 1
    finally:
        env.delenv("VLLM_B200_TUNING_FILE")
        envs.reset_cache()
        tuning_table._table.cache_clear()
        tuning_table._lookup.cache_clear()
