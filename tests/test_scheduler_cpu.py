"""Scheduler policies on the host: the prefill-only second budget of fair chunked prefill and the
pipeline micro-batches' share of the decodes."""

from vllm_cmp170hx_b200.config import CacheConfig, SchedulerConfig
from vllm_cmp170hx_b200.engine.block_pool import make_block_pool
from vllm_cmp170hx_b200.engine.request import Request, SamplingParams
from vllm_cmp170hx_b200.engine.scheduler import ScheduledReq, Scheduler, SchedulerOutput


def _sched(**kw):
    cfg = dict(max_num_seqs=16, max_num_batched_tokens=512, max_model_len=4096, max_num_partial_prefills=2)
    cfg.update(kw)
    return Scheduler(SchedulerConfig(**cfg), CacheConfig(num_blocks=512), make_block_pool(512, 1))


def _decoding(s, n):
    """n requests that finished their prompts and decode."""
    reqs = []
    for i in range(n):
        r = Request(list(range(8)), SamplingParams(max_tokens=50), request_id=f"d{i}")
        s.add(r)
        reqs.append(r)
    out = s.schedule()
    s.update(out, {q.req.request_id: [1] for q in out.reqs})
    return reqs


def test_second_budget_binds_only_while_requests_decode():
    # no decodes: a prompt takes the whole token budget
    s = _sched(prefill_chunk_with_decodes=96)
    s.add(Request(list(range(1000)), SamplingParams(max_tokens=2), request_id="p"))
    assert [q.num_new for q in s.schedule().reqs] == [512]
    # with decodes running: prefill chunks share 96 tokens, decodes are not charged
    s = _sched(prefill_chunk_with_decodes=96)
    _decoding(s, 3)
    s.add(Request(list(range(1000)), SamplingParams(max_tokens=2), request_id="p1"))
    s.add(Request(list(range(1000)), SamplingParams(max_tokens=2), request_id="p2"))
    out = s.schedule()
    got = {q.req.request_id: q.num_new for q in out.reqs}
    assert [got[f"d{i}"] for i in range(3)] == [1, 1, 1]
    assert got["p1"] == 48 and got["p2"] == 48  # split evenly between the two prompts
    # off: the same step gives the prompts the token budget
    s = _sched()
    _decoding(s, 3)
    s.add(Request(list(range(1000)), SamplingParams(max_tokens=2), request_id="p1"))
    got = {q.req.request_id: q.num_new for q in s.schedule().reqs}
    assert got["p1"] == 509


def test_short_prompts_are_not_charged(monkeypatch):
    from vllm_cmp170hx_b200 import envs

    monkeypatch.setenv("VLLM_B200_FAIR_PREFILL_SHORT_BYPASS", "40")
    envs.reset_cache()
    try:
        s = _sched(prefill_chunk_with_decodes=64, max_num_partial_prefills=1)
        _decoding(s, 2)
        s.add(Request(list(range(1000)), SamplingParams(max_tokens=2), request_id="long"))
        s.add(Request(list(range(30)), SamplingParams(max_tokens=2), request_id="short"))
        got = {q.req.request_id: q.num_new for q in s.schedule().reqs}
        assert got["long"] == 64 and got["short"] == 30
    finally:
        envs.reset_cache()


def test_pp_micro_batches_share_the_decodes():
    from types import SimpleNamespace

    from vllm_cmp170hx_b200.engine.runner import ModelRunner

    def req(i, new, start):
        r = Request(list(range(max(start + new, 1))), SamplingParams(max_tokens=4), request_id=f"r{i}")
        return ScheduledReq(r, new, start, True)

    out = SchedulerOutput(reqs=[req(0, 400, 0)] + [req(i, 1, 50) for i in range(1, 7)] + [req(7, 100, 0)])
    for spread, expect_decodes in ((True, [3, 3]), (False, None)):
        fake = SimpleNamespace(st=SimpleNamespace(pp_size=2),
                               cfg=SimpleNamespace(scheduler=SimpleNamespace(pp_spread_decodes=spread)))
        mbs = ModelRunner._micro_batches(fake, out)
        assert sorted(s.req.request_id for mb in mbs for s in mb.reqs) == sorted(s.req.request_id for s in out.reqs)
        if expect_decodes:
            assert [sum(1 for s in mb.reqs if s.num_new == 1) for mb in mbs] == expect_decodes
            assert [sum(s.num_new for s in mb.reqs) for mb in mbs] == [403, 103]
