"""Per-request verify depth (the reference's DSpark adaptive depth, spec_decode/dspark_row_mask*.py):
policy parsing, the E(k) / cost(k) and tau decision rules, the draft-logit statistics, and greedy
speculative decoding under a policy emitting exactly the tokens of plain decoding."""

import json
import math

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_deepseek
from vllm_cmp170hx_b200.engine.depth_policy import DepthPolicy, draft_features, logit_stats
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def _pol(**kw):
    raw = {"schema": "dspark-depth-policy/1", "max_depth": 3, "features": ["bias"],
           "weights": [[0.0], [0.0], [0.0]], "costs": {"1": {"0": 10, "1": 11, "2": 12, "3": 13},
                                                        "4": {"0": 10, "1": 14, "2": 18, "3": 22}}}
    raw.update(kw)
    return DepthPolicy.from_dict(raw)


def test_policy_validation():
    with pytest.raises(ValueError):
        _pol(schema="x")
    with pytest.raises(ValueError):
        _pol(features=["bias", "nope"], weights=[[0, 0]] * 3)
    with pytest.raises(ValueError):
        _pol(costs={"1": {"0": 1, "2": 2}})  # a gap in k
    with pytest.raises(ValueError):
        _pol(costs={"1": {"0": 3, "1": 2}})  # decreasing
    assert _pol().max_depth == 3


def _brute(p, T, b):
    K = len(p)
    best, arg = -1.0, 0
    for k in range(K + 1):
        E = 1 + sum(math.prod(p[:i + 1]) for i in range(k))
        c = T[K] - (T[K] - T[k]) / b
        if E / c >= best - 1e-15:
            best, arg = E / c, k
    return arg


def test_cost_rule_and_interpolation():
    pol = _pol()
    for probs in ([0.9, 0.8, 0.7], [0.1, 0.9, 0.9], [0.5, 0.5, 0.5], [0.99, 0.01, 0.99]):
        p = torch.tensor([probs])
        for b in (1, 2, 4, 7):
            T = pol.cost_row(b, 3)
            assert pol.live(p, b) == [_brute(probs, T, b)], (probs, b)
    # batch 2 lies between the listed 1 and 4: T_2(k) = T_1(k) * 2/3 + T_4(k) / 3
    assert pol.cost_row(2, 3) == pytest.approx([10, 11 * 2 / 3 + 14 / 3, 12 * 2 / 3 + 18 / 3, 13 * 2 / 3 + 22 / 3])


def test_tau_rule():
    pol = _pol(tau={"2": 0.5, "8": 0.2})
    p = torch.tensor([[0.9, 0.6, 0.9], [0.4, 0.9, 0.9]])
    # cumulative products: row 0 .9, .54, .486; row 1 .4, .36, .324
    assert pol.live(p, 2) == [2, 0]
    assert pol.live(p, 8) == [3, 3]  # tau .2
    assert pol.live(p, 5) == [3, 2]  # tau interpolated to .35
    assert pol.live(p[:1], 1) == [_brute([0.9, 0.6, 0.9], pol.cost_row(1, 3), 1)]  # one request: the cost rule


def test_logit_stats_and_features():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 1000, generator=g) * 3
    st = logit_stats(x)
    p = x.softmax(-1)
    assert torch.allclose(st[:, 0], p.max(-1).values, rtol=1e-5)
    assert torch.allclose(st[:, 1], -(p * p.log()).sum(-1), rtol=1e-4)
    f = draft_features(3, 1, st[:, None], torch.full((3, 1), 0.75))
    assert torch.allclose(f[..., 0], torch.ones(3, 1))
    assert torch.allclose(f[..., 1], torch.full((3, 1), math.log(3.0)))


def _cfg(k, policy=""):
    return EngineConfig(model=tiny_deepseek(layers=3, experts=4, hidden=256, vocab=512),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256,
                                                  num_speculative_tokens=k, spec_method="dflash",
                                                  depth_policy=policy),
                        cache=CacheConfig(num_blocks=48), device="cpu", enforce_eager=True)


@pytest.mark.parametrize("bias,cut", [(3.0, False), (-20.0, True)])
def test_greedy_spec_under_depth_policy_matches_plain(tmp_path, bias, cut):
    pstate.set_state(pstate.ParallelState())
    path = tmp_path / "policy.json"
    path.write_text(json.dumps({
        "schema": "dspark-depth-policy/1", "max_depth": 3, "features": ["bias", "logit_conf", "logit_top1", "ent"],
        "weights": [[bias, 0.1, 0.1, -0.01]] * 3,
        "costs": {"1": {"0": 10, "1": 10.5, "2": 11, "3": 11.5}, "4": {"0": 10, "1": 11, "2": 12, "3": 13}}}))
    prompts = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]
    model = HybridForCausalLM(_cfg(0).model, "cpu", seed=3)
    plain = LLM(_cfg(0), model).generate(prompts, SamplingParams(max_tokens=8))
    llm = LLM(_cfg(3, str(path)), model)
    got = llm.generate(prompts, SamplingParams(max_tokens=8))
    model.aux_layer_ids = ()
    assert [o.output_token_ids for o in got] == [o.output_token_ids for o in plain]
    st = llm.engine.runner.spec.stats
    if cut:  # every draft judged not worth verifying: none scheduled
        assert st["proposed"] == 0 and st["depth_cut"] > 0
    else:
        assert st["proposed"] > 0


def test_metrics_lines_report_spec_stats_and_k_histogram():
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine, metrics_lines

    pstate.set_state(pstate.ParallelState())
    cfg = _cfg(3)
    cfg.scheduler.adaptive_k = "by_load"
    model = HybridForCausalLM(cfg.model, "cpu", seed=3)
    eng = LLMEngine(cfg, model)
    eng.add_request([5, 6, 7, 8], SamplingParams(max_tokens=6))
    while eng.has_unfinished() if hasattr(eng, "has_unfinished") else eng.requests:
        eng.step()
    model.aux_layer_ids = ()
    text = "\n".join(metrics_lines(eng))
    assert "b200_spec_draft_tokens_total" in text and 'b200_spec_method{method="dflash"} 1' in text
    assert "b200_adaptive_k_steps{k=" in text


def _stats_worker(rank, world, port, path):
    import datetime
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(9)
        full = torch.randn(5, 1000, generator=g) * 4
        shard = full[:, rank * 500:(rank + 1) * 500]

        def ar(x, op):
            dist.all_reduce(x, op=op)
            return x

        st = logit_stats(shard, ar)
        if rank == 0:
            torch.save((st, logit_stats(full)), path)
    finally:
        dist.destroy_process_group()


def test_logit_stats_over_vocab_shards(tmp_path):
    """Top-1 probability and entropy from two vocab shards (max, normaliser and sum p*logit
    all-reduced) equal the full-vocabulary values."""
    import os

    import torch.multiprocessing as mp

    path = str(tmp_path / "st.pt")
    mp.start_processes(_stats_worker, args=(2, 29900 + os.getpid() % 90, path), nprocs=2, join=True,
                       start_method="spawn")
    sharded, full = torch.load(path)
    assert torch.allclose(sharded, full, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("bias", [3.0, -20.0, 0.0])
def test_row_mask_mode_keeps_the_verify_width_and_matches_plain(tmp_path, bias):
    """depth_mode "mask": every request verifies all k drafts (one verify width, so the verify step's
    CUDA graph applies) and the policy's cut only masks candidates; greedy output equals plain decoding."""
    pstate.set_state(pstate.ParallelState())
    path = tmp_path / "policy.json"
    path.write_text(json.dumps({
        "schema": "dspark-depth-policy/1", "max_depth": 3, "features": ["bias", "logit_conf", "logit_top1", "ent"],
        "weights": [[bias, 0.1, 0.1, -0.01]] * 3,
        "costs": {"1": {"0": 10, "1": 10.5, "2": 11, "3": 11.5}, "4": {"0": 10, "1": 11, "2": 12, "3": 13}}}))
    prompts = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]
    model = HybridForCausalLM(_cfg(0).model, "cpu", seed=3)
    plain = LLM(_cfg(0), model).generate(prompts, SamplingParams(max_tokens=8))
    cfg = _cfg(3, str(path))
    cfg.scheduler.depth_mode = "mask"
    llm = LLM(cfg, model)
    widths = []
    orig = llm.engine.runner.execute

    def spy(out):
        widths.extend(s.num_draft for s in out.reqs if s.num_draft)
        return orig(out)

    llm.engine.runner.execute = spy
    got = llm.generate(prompts, SamplingParams(max_tokens=8))
    model.aux_layer_ids = ()
    assert [o.output_token_ids for o in got] == [o.output_token_ids for o in plain]
    # verify steps keep the full k-draft width (only the length limit near max_tokens narrows one)
    assert widths and widths.count(3) >= len(widths) // 2
    if bias < -10:  # all drafts masked: nothing is a candidate, yet the rows were verified
        assert llm.engine.runner.spec.stats["accepted"] == 0


def _hw_raw(**block):
    hw = {"estimate": "stale", "lag_rounds": 1, "k_choices": [1, 2, 3], "fallback_k": 2, "batch_sizes": [2, 3],
          "t0_ms": {"2": 10.0, "3": 12.0}, "cum_ms": {"2": [0, 1, 2, 3], "3": [0, 1.5, 3, 4.5]},
          "s": {"2": {"1": 1.0, "2": 0.5, "3": 0.5}, "3": {"1": 1.0, "2": 1.0, "3": 1.0}}}
    hw.update(block)
    return {"tau": {"2": 0.3, "3": 0.3}, "host_width": hw}


def _hw_brute(hw, q_rows, b, cap):
    """The objective evaluated term by term, over the K of k_choices at most cap."""
    best = None
    for K in [k for k in hw.k_choices if k <= cap]:
        E, gap = 0.0, 0.0
        for q in q_rows:
            d = max([k for k in range(1, K + 1) if math.prod(q[:k]) >= hw.tau[b]], default=0)
            E += 1 + sum(math.prod(q[:i]) for i in range(1, d + 1))
            gap += hw.cum[b][K] - hw.cum[b][d]
        score = E / (hw.t0[b] + b * hw.cum[b][K] - (1 - hw.share[b][K]) * gap)
        if best is None or score > best[0] + 1e-12:
            best = (score, K)
    return best[1]


def test_host_width_block_parse_and_choice():
    """The policy's host_width block: validation, the K its objective picks (checked against the
    objective evaluated term by term), the fallback for a request without an earlier round, ties to
    the smaller K, and batch sizes outside the block keeping their width."""
    pol = _pol(**_hw_raw())
    hw = pol.host_width
    assert hw is not None and hw.k_choices == (1, 2, 3) and hw.lag == 1
    for bad in ({"estimate": "fresh"}, {"lag_rounds": 0}, {"fallback_k": 5}, {"batch_sizes": [1, 2]},
                {"cum_ms": {"2": [0, 1, 2], "3": [0, 1, 2, 3]}}, {"cum_ms": {"2": [0, 2, 1, 3], "3": [0, 1, 2, 3]}},
                {"s": {"2": {"1": 1.0}, "3": {"1": 1.0, "2": 1.0, "3": 1.0}}}, {"t0_ms": {"2": 0, "3": 1}}):
        with pytest.raises(ValueError):
            _pol(**_hw_raw(**bad))
    gen = torch.Generator().manual_seed(0)
    for _ in range(40):
        b = 2 + int(torch.randint(0, 2, (1,), generator=gen))
        q = torch.rand(b, 3, generator=gen).tolist()
        for cap in (3, 2):
            assert hw.choose(q, b, cap) == _hw_brute(hw, q, b, cap)
    assert hw.choose([[0.9, 0.9, 0.9], None], 2, 3) == 2  # fallback_k
    assert hw.choose([[0.9, 0.9, 0.9]] * 4, 4, 3) is None  # b outside the block
    # every draft below tau: d = 0 for all K, E = 1; the cost grows with K unless shares cancel it
    assert hw.choose([[0.01] * 3] * 3, 3, 3) == 1


def test_host_width_in_the_engine_matches_plain(tmp_path):
    """A policy with a host_width block steers decode steps of two or three requests by their p_i
    rows of the round before; greedy outputs stay those of plain decoding."""
    pstate.set_state(pstate.ParallelState())
    path = tmp_path / "policy.json"
    raw = {"schema": "dspark-depth-policy/1", "max_depth": 3, "features": ["bias", "logit_conf"],
           "weights": [[1.0, 0.2]] * 3,
           "costs": {"1": {"0": 10, "1": 10.5, "2": 11, "3": 11.5}, "4": {"0": 10, "1": 11, "2": 12, "3": 13}}}
    raw.update(_hw_raw())
    path.write_text(json.dumps(raw))
    prompts = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]
    model = HybridForCausalLM(_cfg(0).model, "cpu", seed=3)
    plain = LLM(_cfg(0), model).generate(prompts, SamplingParams(max_tokens=10))
    llm = LLM(_cfg(3, str(path)), model)
    eng = llm.engine
    caps = []
    orig = eng._host_width

    def host_width():
        orig()
        caps.append(eng.scheduler.draft_cap)

    eng._host_width = host_width
    got = llm.generate(prompts, SamplingParams(max_tokens=10))
    model.aux_layer_ids = ()
    assert [o.output_token_ids for o in got] == [o.output_token_ids for o in plain]
    spec = eng.runner.spec
    assert spec.depth.host_width is not None and caps and all(1 <= c <= 3 for c in caps)
    assert not spec.p_rounds  # finished requests' rows are dropped
