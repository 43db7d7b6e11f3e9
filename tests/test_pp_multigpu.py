"""Pipeline parallelism on 2 GPUs (NCCL over NVLink, NVLS off): the tiny models generate the same greedy
tokens at PP=2 as on one GPU, through the CUDA kernels -- packed hidden / residual hops between the
stages, verify results and drafts broadcast from the last stage, and the two draft transports: the
split draft event (drafts waited for only before the first stage's forward) and the DFlash draft tail
(the lm_head and picks on the first stage)."""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(9 + 13 * i)] for i in range(3)]


def _generate(pp: int, method: str):
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig, tiny, \
        tiny_deepseek
    from vllm_cmp170hx_b200.engine.llm_engine import LLM
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM

    if method == "mtp":  # Marlin experts, fp8 attention projections, one MTP layer
        m = tiny_deepseek(layers=2, experts=4, hidden=256, vocab=512)
        m.moe.intermediate = 256
    else:  # EXL3 experts, the DFlash block drafter over auxiliary hidden states
        m = tiny(layers=4, experts=4, hidden=256, expert_format="exl3")
        m.moe.intermediate = 256
        m.moe.shared_intermediate = 256
    cfg = EngineConfig(model=m, parallel=ParallelConfig(pipeline_parallel_size=pp),
                       scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256,
                                                 num_speculative_tokens=2, spec_method=method),
                       cache=CacheConfig(num_blocks=32), device="cuda", enforce_eager=True)
    model = HybridForCausalLM(cfg.model, "cuda", seed=5, init_mode="sliced")
    outs = LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=8))
    return [o.output_token_ids for o in outs]


def _worker(rank, world, port, q, method, env):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0", **env)
    from vllm_cmp170hx_b200 import _ext
    from vllm_cmp170hx_b200.engine.runner import ModelRunner
    from vllm_cmp170hx_b200.parallel import state as pstate

    try:
        st = pstate.init(tp_size=1, pp_size=world, timeout_s=60)
        toks = _generate(world, method)
        _ext.check_status(st.device)
        q.put((rank, (toks, ModelRunner.split_draft_events, ModelRunner.draft_tail_steps)))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, repr(e) + traceback.format_exc()))
    finally:
        pstate.destroy()


def _single(q, method):
    try:
        q.put(_generate(1, method))
    except Exception as e:  # noqa: BLE001
        q.put(repr(e))


def _spawn(target, n, args, port=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=((r, n, port, q) if port else (q,)) + args) for r in range(n)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return res


def _close(a: list, b: list) -> int:
    """Sequences whose greedy tokens differ (a near-tie in the tiny random model's router may flip on a
    different rounding of a micro-batch's GEMM)."""
    return sum(x != y for x, y in zip(a, b))


@pytest.mark.parametrize("method,env", [("mtp", {}), ("mtp", {"VLLM_B200_PP_SPLIT_DRAFTS": "1"}),
                                        ("dflash", {}), ("dflash", {"VLLM_B200_PP_DRAFT_TAIL_STAGE": "0"})])
def test_pp2_matches_one_gpu(method, env):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    (ref,) = _spawn(_single, 1, (method,))
    assert not isinstance(ref, str), ref
    port = 26700 + os.getpid() % 300 + 7 * len(env) + (3 if method == "dflash" else 0)
    res = dict(_spawn(_worker, 2, (method, env), port=port))
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    toks, split_events, tail_steps = res[0]
    assert toks == res[1][0]  # every stage stores the same outputs
    assert all(len(t) == 8 for t in toks)
    assert _close(toks, ref) <= 1, (toks, ref)
    if "VLLM_B200_PP_SPLIT_DRAFTS" in env:
        assert split_events > 0
    if "VLLM_B200_PP_DRAFT_TAIL_STAGE" in env:
        assert tail_steps > 0
