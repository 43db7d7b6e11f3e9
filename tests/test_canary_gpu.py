"""Canary-guarded outputs of the hot kernels on shapes that end mid-tile: every kernel writes its rows and
nothing around them (guard rows before and after, guard tails after each row where the op takes a row
stride), and the results equal those of an unguarded call.  Also: a decode forward of the tiny hybrid
model makes no host synchronisation (the property its CUDA-graph capture relies on)."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext, ops
from vllm_cmp170hx_b200.utils.canary import CanaryError, Guarded

pytestmark = pytest.mark.gpu


def test_canary_detects_a_stray_write():
    g = Guarded((5, 64), torch.bfloat16, "cuda", row_pad=8)
    g.view.fill_(1.0)
    g.check()
    g.buf[2 + g.pad, 64] = 0  # one element past a row's end
    with pytest.raises(CanaryError, match="row guard tails"):
        g.check()


@pytest.mark.parametrize("M,N,K", [(1, 256, 256), (37, 2304, 512), (129, 384, 2304), (300, 4096, 256)])
def test_gemm_writes_only_its_output(M, N, K):
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16() * K ** -0.5
    ref = ops.gemm(x, w)
    for row_pad in (0, 8):
        g = Guarded((M, N), torch.bfloat16, "cuda", row_pad=row_pad)
        ops.gemm(x, w, out=g.view)
        torch.cuda.synchronize()
        g.check()
        assert torch.equal(g.view, ref)


def test_norm_silu_gate_and_attention_write_only_their_outputs():
    from vllm_cmp170hx_b200.ops import gqa as gqa_ops

    T, H = 45, 768
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    g = Guarded((T, H), torch.bfloat16, "cuda")
    ops.rms_norm(x, w, 1e-6, out=g.view)
    torch.cuda.synchronize()
    g.check()
    gu = torch.randn(T, 2 * H, device="cuda").bfloat16()
    g = Guarded((T, H), torch.bfloat16, "cuda")
    ops.silu_mul(gu, out=g.view)
    torch.cuda.synchronize()
    g.check()
    # engram gate accumulates into its output in place: the guards around it stay intact
    kv = torch.randn(T, 2 * H, device="cuda").bfloat16()
    g = Guarded((T, H), torch.bfloat16, "cuda", row_pad=8)
    g.view.zero_()
    _ext.ops().engram_gate(x, kv, w, w, 1e-6, g.view)
    torch.cuda.synchronize()
    g.check()
    # dense grouped-query attention: 3 sequences, 2 key-value heads of 4 query heads each
    nkv, G, lens = 2, 4, [1, 70, 200]
    Tq = sum(lens)
    nb = sum((n + 63) // 64 for n in lens)
    cache = torch.randn(nb * 64 * nkv, 512, device="cuda").bfloat16()
    q = torch.randn(Tq * nkv, G, 512, device="cuda").bfloat16()
    q[..., 256:] = 0
    bt = torch.zeros(3, 4, dtype=torch.int32)
    b = 0
    pos, seq = [], []
    for s, n in enumerate(lens):
        for j in range((n + 63) // 64):
            bt[s, j] = b
            b += 1
        pos += list(range(n))
        seq += [s] * n
    ctx = torch.tensor(pos, dtype=torch.int32, device="cuda") + 1
    tseq = torch.tensor(seq, dtype=torch.int32, device="cuda")
    ref = gqa_ops.attention(q, cache, ctx, tseq, bt.cuda(), nkv, max(lens), splits=1)
    for splits in (1, 3):
        g = Guarded((Tq * nkv, G, 512), torch.bfloat16, "cuda")
        gqa_ops.attention(q, cache, ctx, tseq, bt.cuda(), nkv, max(lens), out=g.view, splits=splits)
        torch.cuda.synchronize()
        g.check()
        assert (g.view[..., 256:].float() - ref[..., 256:].float()).abs().max() < 2e-2


def test_decode_forward_makes_no_host_sync():
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.engine.request import SamplingParams
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = EngineConfig(model=tiny(layers=4, experts=8), scheduler=SchedulerConfig(max_num_seqs=4, max_model_len=512),
                       cache=CacheConfig(num_blocks=32), device="cuda", enforce_eager=True)
    eng = LLMEngine(cfg)
    for i in range(3):
        eng.add_request(list(range(5 + i, 50 + i)), SamplingParams(max_tokens=4))
    eng.step()  # prefill
    out = eng.scheduler.schedule()
    assert out.decode_only
    h = eng.runner._host_inputs(out)
    d, ctx, _ = eng.runner._context(h)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        with torch.inference_mode():
            eng.runner.model(d["ids"], ctx)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
