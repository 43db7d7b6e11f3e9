"""Block-diagonal (grouped) projection: output group g is input group g times W_g^T, for bf16 and
fp8 block-scaled groups, against the dense block-diagonal matrix product."""

import pytest
import torch

from vllm_cmp170hx_b200.formats import fp8 as f8
from vllm_cmp170hx_b200.models.layers import GroupedLinear


def _ref(x, w, fmt):
    G = w.shape[0]
    if fmt == "fp8_block":
        w = torch.stack([f8.dequantize(*f8.quantize(w[g].float())) for g in range(G)])
    return torch.cat([x[:, g].float() @ w[g].float().t() for g in range(G)], dim=-1)


def _case(T, G, out_g, in_g, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, G, in_g, generator=g).to(torch.bfloat16)
    w = (torch.randn(G, out_g, in_g, generator=g) * in_g ** -0.5).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("fmt", ["bf16", "fp8_block"])
def test_grouped_linear_cpu(fmt):
    x, w = _case(5, 4, 128, 256, 0)
    y = GroupedLinear(w, fmt)(x)
    r = _ref(x, w, fmt)
    assert y.shape == (5, 4 * 128)
    assert ((y.float() - r).norm() / r.norm()).item() < 1e-2


def test_grouped_linear_rejects_bad_input():
    x, w = _case(2, 4, 128, 256, 1)
    with pytest.raises(ValueError):
        GroupedLinear(w)(x[:, :3])


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["bf16", "fp8_block"])
@pytest.mark.parametrize("T", [1, 37, 200])
def test_grouped_linear_gpu(fmt, T):
    from vllm_cmp170hx_b200 import _ext

    x, w = _case(T, 8, 128, 512, T)
    layer = GroupedLinear(w.cuda(), fmt)
    y = layer(x.cuda())
    torch.cuda.synchronize()
    _ext.check_status(torch.device("cuda"))
    r = _ref(x, w, fmt)
    assert ((y.float().cpu() - r).norm() / r.norm()).item() < 1e-2
