"""Tensor parallel on CPU ranks (gloo): the tiny hybrid model at TP=2 with
sliced weights generates the same greedy tokens as at TP=1 (heads, expert
intermediates and the vocab shard split across ranks; per-rank sampling
winners combined)."""

import json
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from vllm_cmp170hx_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig, tiny, tiny_deepseek,
                                       tiny_dsv4)

PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(9 + 13 * i)] for i in range(3)]


def _cfg(tp, fmt, pp=1):
    k = 0
    hc = fmt.endswith("_hc")
    fmt = fmt[:-3] if hc else fmt
    ep = fmt.endswith("_ep")
    fmt = fmt[:-3] if ep else fmt
    method = "mtp"
    if fmt == "exl3_dflash":  # DFlash block drafter (auxiliary hidden states cross the pipeline hop)
        fmt, method, k = "exl3", "dflash", 2
    if fmt == "dsv4":  # DeepSeek-V4.1 attention (window + compressed groups + sinks), delayed mHC, EXL3
        m = tiny_dsv4(layers=3, experts=4, hidden=256, vocab=512)
    elif fmt == "deepseek_mtp":  # Marlin experts, fp8 attention projections, MTP speculative decoding
        m = tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512)
        m.moe.intermediate = 256
        m.mla.num_heads = 4  # two heads per rank: q_b shards of 384 rows hold whole fp8 scale blocks
        k = 2
    else:
        m = tiny(layers=4, experts=4, hidden=256, expert_format=fmt)
        m.moe.intermediate = 256  # two H128 blocks: one per rank at TP=2
        m.moe.shared_intermediate = 256
        m.hc_mult = 4 if hc else 0
    return EngineConfig(model=m, parallel=ParallelConfig(tensor_parallel_size=tp, expert_parallel=ep,
                                                         pipeline_parallel_size=pp),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=32, max_model_len=256,
                                                  num_speculative_tokens=k, spec_method=method),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


def _generate(tp, fmt, pp=1):
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM

    from vllm_cmp170hx_b200.parallel import state as pstate

    cfg = _cfg(tp, fmt, pp)
    pstate.get().expert_parallel = cfg.parallel.expert_parallel
    model = HybridForCausalLM(cfg.model, "cpu", seed=5, init_mode="sliced")
    outs = LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=6 if cfg.scheduler.num_speculative_tokens else 3))
    return [o.output_token_ids for o in outs]


def _worker(rank, world, port, fmt, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.init(tp_size=world, device="cpu", timeout_s=120)
    toks = _generate(world, fmt)
    if rank == 0:
        with open(path, "w") as f:
            json.dump(toks, f)
    pstate.destroy()


@pytest.mark.parametrize("fmt", ["bf16", "exl3", "deepseek_mtp", "exl3_ep", "deepseek_mtp_ep", "exl3_hc", "dsv4"])
def test_tp2_matches_tp1(fmt):
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    ref = _generate(1, fmt)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.json")
        port = 29500 + os.getpid() % 1000
        mp.start_processes(_worker, args=(2, port, fmt, path), nprocs=2, join=True, start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    assert got == ref


def _pp_worker(rank, world, port, fmt, tp, path, env=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), **(env or {}))
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.init(tp_size=tp, pp_size=world // tp, device="cpu", timeout_s=120)
    toks = _generate(tp, fmt, world // tp)
    if rank == 0:
        from vllm_cmp170hx_b200.engine.runner import ModelRunner

        with open(path, "w") as f:
            json.dump({"tokens": toks, "split_events": ModelRunner.split_draft_events,
                       "tail_steps": ModelRunner.draft_tail_steps} if env else toks, f)
    pstate.destroy()


@pytest.mark.parametrize("fmt,tp", [("exl3", 1), ("deepseek_mtp", 1), ("deepseek_mtp", 2), ("exl3_hc", 1),
                                    ("exl3_dflash", 1), ("dsv4", 1)])
def test_pp2_matches_pp1(fmt, tp):
    """Two pipeline stages (packed p2p hops, micro-batches, token / draft broadcast from the last
    stage) generate the same tokens as one stage; deepseek_mtp adds MTP speculative decoding, exl3_hc
    hyper-connection streams (the whole mHC state crosses the stage boundary)."""
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    ref = _generate(1, fmt)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.json")
        port = 28700 + os.getpid() % 1000
        mp.start_processes(_pp_worker, args=(2 * tp, port, fmt, tp, path), nprocs=2 * tp, join=True,
                           start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    assert got == ref


@pytest.mark.parametrize("fmt", ["deepseek_mtp", "exl3_dflash"])
def test_pp2_split_draft_event_matches_pp1(fmt):
    """Split draft event: the last stage's drafts travel by an asynchronous broadcast that the first
    stage waits for only before its next forward; the other stages schedule on draft counts alone.
    Greedy outputs equal one stage's, and the asynchronous path ran."""
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    ref = _generate(1, fmt)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.json")
        port = 29700 + os.getpid() % 1000
        mp.start_processes(_pp_worker, args=(2, port, fmt, 1, path, {"VLLM_B200_PP_SPLIT_DRAFTS": "1"}), nprocs=2,
                           join=True, start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    assert got["tokens"] == ref and got["split_events"] > 0


def test_pp2_draft_tail_on_first_stage_matches_pp1():
    """Pipeline draft tail: the last stage runs the DFlash block forward and sends its hidden states
    to stage 0, which holds a copy of the lm_head shard, picks the drafts and roots their broadcast.
    Greedy outputs equal one stage's, and the tail ran on stage 0."""
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    ref = _generate(1, "exl3_dflash")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.json")
        port = 30700 + os.getpid() % 1000
        mp.start_processes(_pp_worker, args=(2, port, "exl3_dflash", 1, path, {"VLLM_B200_PP_DRAFT_TAIL_STAGE": "0"}),
                           nprocs=2, join=True, start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    assert got["tokens"] == ref and got["tail_steps"] > 0


@pytest.mark.parametrize("fmt", ["exl3", "deepseek_mtp"])
def test_emulated_tp_runs_per_rank_shapes(fmt):
    """One process standing in for rank 0 of a TP=2 group: the engine builds the per-rank shards and
    steps through them with collectives returning local data (per-rank kernel profiling)."""
    from vllm_cmp170hx_b200.parallel import state as pstate

    st = pstate.emulate(2, device="cpu")
    try:
        toks = _generate(2, fmt)
        assert [len(t) for t in toks] == [6 if fmt == "deepseek_mtp" else 3] * len(PROMPTS)
        assert st.emulated and pstate.get().tp_size == 2
    finally:
        pstate.set_state(pstate.ParallelState())


def _sp_worker(rank, world, port, fmt, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.init(tp_size=world, device="cpu", timeout_s=120)
    cfg = _cfg(world, fmt)
    pstate.get().expert_parallel = True
    model = HybridForCausalLM(cfg.model, "cpu", seed=5, init_mode="sliced")
    calls = {"sp": 0}
    orig = HybridForCausalLM._forward_sp

    def counted(self, *a, **k):
        calls["sp"] += 1
        return orig(self, *a, **k)

    HybridForCausalLM._forward_sp = counted
    outs = LLM(cfg, model).generate(SP_PROMPTS, SamplingParams(max_tokens=4))
    if rank == 0:
        with open(path, "w") as f:
            json.dump({"toks": [o.output_token_ids for o in outs], "sp_steps": calls["sp"]}, f)
    pstate.destroy()


SP_PROMPTS = [[(7 * i + 5 * j) % 500 for j in range(6 + 3 * i)] for i in range(4)]


@pytest.mark.parametrize("fmt", ["exl3_ep", "bf16_ep"])
def test_sequence_parallel_ep_matches_tp1(fmt):
    """Expert parallel at TP=2 in the sequence-parallel layout (token-sharded residual stream: all-gather
    before attention, reduce-scatter after it, dispatch to the experts' ranks and combine back), over
    torch.distributed on gloo: the same greedy tokens as one rank, with the layout actually taken by
    the steps whose token count divides over the ranks."""
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = _cfg(1, fmt)
    model = HybridForCausalLM(cfg.model, "cpu", seed=5, init_mode="sliced")
    ref = [o.output_token_ids for o in LLM(cfg, model).generate(SP_PROMPTS, SamplingParams(max_tokens=4))]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.json")
        port = 27300 + os.getpid() % 1000
        mp.start_processes(_sp_worker, args=(2, port, fmt, path), nprocs=2, join=True, start_method="spawn")
        with open(path) as f:
            got = json.load(f)
    assert got["sp_steps"] >= 3, got
    assert got["toks"] == ref
