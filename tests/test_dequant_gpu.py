"""Marlin int4 experts and fp8 block-scaled linears (tcgen05 dequant GEMM) vs
their format oracles."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext
from vllm_cmp170hx_b200.formats import fp8 as f8
from vllm_cmp170hx_b200.formats import marlin as fm
from vllm_cmp170hx_b200.ops import dequant
from vllm_cmp170hx_b200.oracle import moe as moe_ref

pytestmark = pytest.mark.gpu


def _rel(y, r):
    return ((y.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,E,k", [(3, 8, 2), (64, 16, 4), (300, 4, 2)])
def test_marlin_moe(T, E, k):
    g = torch.Generator().manual_seed(T)
    H, I = 256, 384
    gp, gs = fm.random_experts(E, H, I, generator=g)
    up, us = fm.random_experts(E, H, I, generator=g)
    dp, ds = fm.random_experts(E, I, H, generator=g)
    ex = dequant.MarlinExperts(gp, gs, up, us, dp, ds, H, I)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids, w = moe_ref.topk(torch.randn(T, E, generator=g), k, 0)
    ref = dequant.marlin_moe(x, ids, w, ex, out_f32=True)
    exg = dequant.MarlinExperts(*(t.cuda() for t in (gp, gs, up, us, dp, ds)), H, I)
    y = dequant.marlin_moe(x.cuda(), ids.cuda(), w.cuda(), exg, out_f32=True)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 1e-2, _rel(y.cpu(), ref)


@pytest.mark.parametrize("T,N,K", [(1, 256, 512), (37, 384, 1024), (200, 1536, 768)])
def test_fp8_block_linear(T, N, K):
    g = torch.Generator().manual_seed(N)
    q, s = f8.random_weight(N, K, 0.05, generator=g)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    ref = x.float() @ f8.dequantize(q, s).t()
    y = dequant.fp8_linear(x.cuda(), dequant.Fp8Linear(q.cuda(), s.cuda()))
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 1e-2, _rel(y.cpu(), ref)


@pytest.mark.parametrize("first,count", [(0, 4), (12, 4)])
def test_marlin_moe_expert_subset(first, count):
    """Expert parallel: experts [first, first + count) of 16 on this rank, the rest dropped."""
    T, E, k = 80, 16, 4
    g = torch.Generator().manual_seed(first + 7)
    H, I = 256, 256
    gp, gs = fm.random_experts(E, H, I, generator=g)
    up, us = fm.random_experts(E, H, I, generator=g)
    dp, ds = fm.random_experts(E, I, H, generator=g)
    ex = dequant.MarlinExperts(gp, gs, up, us, dp, ds, H, I).select(first, count)
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[first:first + count] = torch.arange(count, dtype=torch.int32)
    ex.expert_map = emap
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids, w = moe_ref.topk(torch.randn(T, E, generator=g), k, 0)
    ref = dequant.marlin_moe(x, ids, w, ex, out_f32=True)
    exg = dequant.MarlinExperts(*(getattr(ex, f).cuda() for f in ("gate", "gate_s", "up", "up_s", "down", "down_s")),
                                H, I, expert_map=emap.cuda())
    y = dequant.marlin_moe(x.cuda(), ids.cuda(), w.cuda(), exg, out_f32=True)
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    assert _rel(y.cpu(), ref) < 1e-2, _rel(y.cpu(), ref)
