"""Engram memory of the DeepSeek-V4.1-style model on CPU: the gate against a direct evaluation of its
definition, and the model with an Engram layer in the engine (generation independent of prompt
chunking, greedy MTP speculative decoding equal to plain decoding, an unreadable table row finishing
only the requests that used it)."""

import numpy as np
import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny_dsv4
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.engram import gate_ref
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.parallel import state as pstate


def test_gate_matches_definition():
    torch.manual_seed(0)
    T, H = 3, 64
    a, h = torch.randn(T, H), torch.randn(T, H)
    kv = torch.randn(T, 2 * H)
    wh, wk = 1 + 0.1 * torch.randn(H), 1 + 0.1 * torch.randn(H)
    got = gate_ref(a, h, kv, wh, wk, 1e-6)
    for t in range(T):
        hn = h[t] / torch.sqrt((h[t] ** 2).mean() + 1e-6) * wh
        k = kv[t, :H]
        kn = k / torch.sqrt((k ** 2).mean() + 1e-6) * wk
        alpha = 1 / (1 + torch.exp(-(hn @ kn) / H ** 0.5))
        assert torch.allclose(got[t], a[t] + alpha * kv[t, H:], atol=1e-5)


PROMPTS = [[(5 * i + 3 * j) % 500 for j in range(n)] for i, n in enumerate([9, 40, 71])]


def _cfg(budget, k=0):
    m = tiny_dsv4(layers=3, engram=True)
    m.num_mtp_layers = 1 if k else 0
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=budget,
                                                           max_model_len=256, num_speculative_tokens=k),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


@pytest.fixture(scope="module")
def model():
    pstate.set_state(pstate.ParallelState())
    return HybridForCausalLM(_cfg(32).model, "cpu", seed=5)


def _gen(model, cfg, n=6):
    return [o.output_token_ids for o in LLM(cfg, model).generate(PROMPTS, SamplingParams(max_tokens=n))]


def test_engram_layer_changes_the_output(model):
    assert model.engram is not None and model.layer(1).engram is not None
    plain = tiny_dsv4(layers=3)
    other = HybridForCausalLM(plain, "cpu", seed=5)
    a = _gen(model, _cfg(64))
    cfg = _cfg(64)
    cfg.model = plain
    b = [o.output_token_ids for o in LLM(cfg, other).generate(PROMPTS, SamplingParams(max_tokens=6))]
    assert a != b


def test_engram_generation_independent_of_chunking(model):
    assert _gen(model, _cfg(16)) == _gen(model, _cfg(128))


def test_engram_greedy_mtp_spec_matches_plain(model):
    plain = _gen(model, _cfg(64))
    llm = LLM(_cfg(64, k=2), model)
    assert [o.output_token_ids for o in llm.generate(PROMPTS, SamplingParams(max_tokens=6))] == plain


def test_unreadable_row_fails_only_its_requests(model, tmp_path):
    """The table file is cut before its last row, and the n-grams holding a sentinel token (only in the
    first prompt) are routed to that row: its reads fail after the retries, the row turns NaN and only
    the first request finishes with an error."""
    from vllm_cmp170hx_b200.storage import tables

    mem = model.engram
    last = mem.heads * mem.vocab - 1
    sentinel = 499
    path = str(tmp_path / "engram.bin")
    np.fromfile(mem.path, dtype=np.uint8)[:last * tables.row_bytes(mem.dim)].tofile(path)
    old_table, old_ids = mem.table, mem.ids_of

    def ids_of(tokens, positions):
        ids = old_ids(tokens, positions)
        toks = np.asarray(tokens)
        hit = np.array([sentinel in toks[max(0, p - 1):p + 1] for p in positions])
        ids[hit, 0] = last
        return ids

    mem.table = tables.RowTable(path, last + 1, mem.dim, retries=1)
    mem.ids_of = ids_of
    prompts = [[sentinel] + PROMPTS[0], PROMPTS[1], PROMPTS[2]]
    try:
        outs = LLM(_cfg(64), model).generate(prompts, SamplingParams(max_tokens=4))
    finally:
        mem.table, mem.ids_of = old_table, old_ids
    assert outs[0].finish_reason == "error"
    assert all(o.finish_reason != "error" and len(o.output_token_ids) == 4 for o in outs[1:])
    assert all(sentinel not in o.output_token_ids for o in outs[1:])
