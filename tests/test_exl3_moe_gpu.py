"""EXL3 dense linear and routed-expert kernels (tcgen05) vs the fp32 oracle."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.formats import exl3 as fx
from vllm_cmp170hx_b200.ops import moe as moe_ops
from vllm_cmp170hx_b200.oracle import moe as moe_ref

pytestmark = pytest.mark.gpu


def _rel(y, r):
    return ((y.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("bits_x2,codebook", [(8, 2), (8, 1), (4, 2), (6, 1), (5, 2)])
@pytest.mark.parametrize("T", [1, 13, 200])
def test_exl3_linear(bits_x2, codebook, T):
    g = torch.Generator().manual_seed(bits_x2 * 10 + codebook)
    m = fx.random_matrix(512, 384, bits_x2, codebook, generator=g)
    x = torch.randn(T, 512, generator=g).to(torch.bfloat16)
    ref = fx.linear(x.float(), m)
    y = moe_ops.exl3_linear(x.cuda(), m.to("cuda"), out_dtype=torch.float32)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 2e-3, _rel(y.cpu(), ref)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_topk(mode):
    torch.manual_seed(mode)
    logits = torch.randn(77, 256)
    bias = torch.randn(256) * 0.1 if mode else None
    ids_r, w_r = moe_ref.topk(logits, 8, mode, bias, 2.5)
    ids, w = moe_ops.topk(logits.cuda(), 8, mode, None if bias is None else bias.cuda(), 2.5)
    assert torch.equal(ids.cpu(), ids_r)
    assert torch.allclose(w.cpu(), w_r, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T,E,k", [(4, 16, 4), (64, 32, 8), (300, 8, 2), (512, 16, 8), (1024, 8, 4)])
def test_exl3_moe(T, E, k):
    g = torch.Generator().manual_seed(T + E)
    H, I = 256, 384
    gate = [fx.random_matrix(H, I, 8, 2, generator=g) for _ in range(E)]
    up = [fx.random_matrix(H, I, 8, 2, generator=g) for _ in range(E)]
    down = [fx.random_matrix(I, H, 8, 2, generator=g) for _ in range(E)]
    ex = moe_ops.Exl3Experts.from_matrices(gate, up, down)
    x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    ids, w = moe_ref.topk(logits, k, 0)
    ref = moe_ref.exl3_experts(x.float(), ids, w, {"gate": gate, "up": up, "down": down}, None, {})
    y = moe_ops.exl3_moe(x.cuda(), ids.cuda(), w.cuda(), ex.to("cuda"), out_f32=True)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 5e-3, _rel(y.cpu(), ref)
    # deterministic run to run
    y2 = moe_ops.exl3_moe(x.cuda(), ids.cuda(), w.cuda(), ex.to("cuda"), out_f32=True)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("first,count", [(0, 4), (12, 4), (5, 9)])
def test_exl3_moe_expert_subset(first, count):
    """Expert parallel: this rank holds experts [first, first + count); assignments to the others are
    dropped (the rows past the local ones stay unused), and the output is the local experts' share."""
    T, E, k = 96, 16, 8
    g = torch.Generator().manual_seed(first * 31 + count)
    H, I = 256, 256
    gate = [fx.random_matrix(H, I, 8, 2, generator=g) for _ in range(E)]
    up = [fx.random_matrix(H, I, 8, 2, generator=g) for _ in range(E)]
    down = [fx.random_matrix(I, H, 8, 2, generator=g) for _ in range(E)]
    sl = slice(first, first + count)
    ex = moe_ops.Exl3Experts.from_matrices(gate[sl], up[sl], down[sl])
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[sl] = torch.arange(count, dtype=torch.int32)
    ex.expert_map = emap
    x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16)
    ids, w = moe_ref.topk(torch.randn(T, E, generator=g), k, 0)
    ref = moe_ref.exl3_experts(x.float(), ids, w, {"gate": gate[sl], "up": up[sl], "down": down[sl],
                                                   "expert_map": emap}, None, {})
    y = moe_ops.exl3_moe(x.cuda(), ids.cuda(), w.cuda(), ex.to("cuda"), out_f32=True)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 5e-3, _rel(y.cpu(), ref)
