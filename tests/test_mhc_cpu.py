"""Manifold-constrained hyper-connections on CPU: the oracle's algebra (Sinkhorn tends to a doubly
stochastic mix, identity post keeps the streams, one-hot collapse picks a stream) and hybrid models
with hc streams (immediate and delayed) stepping through the engine."""

import pytest
import torch

from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
from vllm_cmp170hx_b200.engine.llm_engine import LLM
from vllm_cmp170hx_b200.engine.request import SamplingParams
from vllm_cmp170hx_b200.models.hybrid import HybridForCausalLM
from vllm_cmp170hx_b200.oracle import mhc as ref
from vllm_cmp170hx_b200.parallel import state as pstate


def _params(n, d, g):
    N = 2 * n + n * n
    return (torch.randn(N, n * d, generator=g) * (n * d) ** -0.5, torch.rand(3, generator=g) + 0.5,
            torch.rand(N, generator=g) - 0.5)


def test_sinkhorn_is_doubly_stochastic():
    g = torch.Generator().manual_seed(0)
    n, d = 4, 64
    H = torch.randn(5, n, d, generator=g).to(torch.bfloat16)
    fn, scale, base = _params(n, d, g)
    pre, post, comb = ref.coefficients(H, fn, scale, base, 1e-6, 1e-6, 2.0, 20)
    assert torch.allclose(comb.sum(-2), torch.ones(5, n), atol=1e-4)
    assert torch.allclose(comb.sum(-1), torch.ones(5, n), atol=1e-2)
    assert (pre > 0).all() and (pre < 1 + 1e-5).all() and (post > 0).all() and (post < 2).all()


def test_identity_post_and_one_hot_collapse():
    g = torch.Generator().manual_seed(1)
    n, d = 4, 32
    H = torch.randn(3, n, d, generator=g).to(torch.bfloat16)
    x = torch.randn(3, d, generator=g).to(torch.bfloat16)
    same = ref.apply_post(x, H, torch.zeros(3, n), torch.eye(n).expand(3, n, n))
    assert torch.equal(same, H)
    w = torch.ones(d, dtype=torch.bfloat16)
    onehot = torch.zeros(3, n)
    onehot[:, 2] = 1.0
    assert torch.allclose(ref.collapse_norm(H, onehot, w, 1e-6).float(), ref.collapse_norm(H[:, 2:3], None, w, 1e-6).float())


def _cfg(delayed):
    m = tiny(layers=3, experts=4, hidden=256, expert_format="bf16")
    m.hc_mult, m.hc_delayed = 4, delayed
    return EngineConfig(model=m, scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256),
                        cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)


@pytest.mark.parametrize("delayed", [False, True])
def test_hc_model_generates(delayed):
    pstate.set_state(pstate.ParallelState())
    cfg = _cfg(delayed)
    model = HybridForCausalLM(cfg.model, "cpu", seed=2)
    prompts = [[(3 * i + 7 * j) % 500 for j in range(5 + 9 * i)] for i in range(3)]
    outs = [o.output_token_ids for o in LLM(cfg, model).generate(prompts, SamplingParams(max_tokens=5))]
    again = [o.output_token_ids for o in LLM(cfg, model).generate(prompts, SamplingParams(max_tokens=5))]
    assert outs == again and all(len(o) == 5 for o in outs)
    # the streams matter: the same weights without hyper-connections decode differently
    assert model.layers[0].hc_attn.fn.shape == (2 * 4 + 16, 4 * 256)


@pytest.mark.parametrize("delayed", [False, True])
def test_hc_state_hop_round_trip(delayed):
    """The mHC state packed into one 16-byte-aligned uint8 message and back (pipeline hop)."""
    from vllm_cmp170hx_b200.config import tiny
    from vllm_cmp170hx_b200.models import hybrid

    cfg = tiny(layers=2, experts=4, hidden=256)
    cfg.hc_mult, cfg.hc_delayed = 4, delayed
    T, n, d = 5, 4, 256
    st = hybrid.HCState(torch.randn(T, d).bfloat16(), torch.randn(T, n, d).bfloat16(), torch.rand(T, n),
                        torch.rand(T, n, n), torch.rand(T, n) if delayed else None)
    buf = hybrid.hc_pack(st, cfg)
    assert buf.dtype == torch.uint8 and buf.numel() == hybrid.hc_hop_bytes(cfg, T) and buf.numel() % 16 == 0
    back = hybrid.hc_unpack(buf.clone(), cfg, T)
    for name in ("x", "H", "post", "comb"):
        assert torch.equal(getattr(back, name), getattr(st, name)), name
    assert (back.pre_mix is None) == (not delayed)
    if delayed:
        assert torch.equal(back.pre_mix, st.pre_mix)
