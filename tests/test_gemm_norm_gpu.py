"""tcgen05 bf16 GEMM and RMSNorm kernels vs fp32 PyTorch references."""

import pytest
import torch

from vllm_cmp170hx_b200 import _ext, ops
from vllm_cmp170hx_b200.oracle import basic as ref

pytestmark = pytest.mark.gpu


def _rel_err(y, r):
    return ((y.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12)).item()


def _tile_max_err(y, r, tm=128, tn=16):
    """Worst tile of the output: max |y - r| over a tile against the tile's max |r| (a wrong tile in a
    large matrix barely moves the global norm error)."""
    y, r = y.float(), r.float()
    worst = 0.0
    for i in range(0, r.shape[0], tm):
        for j in range(0, r.shape[1], tn):
            d = (y[i:i + tm, j:j + tn] - r[i:i + tm, j:j + tn]).abs().max().item()
            worst = max(worst, d / max(r[i:i + tm, j:j + tn].abs().max().item(), 1e-6))
    return worst


@pytest.mark.parametrize("M,N,K", [(1, 2304, 2304), (7, 4096, 2304), (16, 256, 128), (33, 1000, 520),
                                   (128, 2304, 4096), (129, 512, 256), (300, 777, 1024), (1024, 2048, 2304)])
def test_gemm_bf16(M, N, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    y = ops.gemm(x, w)
    r = x.float() @ w.float().t()
    torch.cuda.synchronize()
    _ext.check_status(x.device)
    assert _rel_err(y, r) < 1e-2, (M, N, K, _rel_err(y, r))
    # both tile orientations of the kernel (swapped for M <= 128: tokens along the tile's N)
    assert _tile_max_err(y, r) < 3e-2, (M, N, K, _tile_max_err(y, r))
    assert _tile_max_err(y, r, 16, 128) < 3e-2, (M, N, K)


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_gemm_bf16_splits_and_bias(splits):
    torch.manual_seed(1)
    M, N, K = 24, 640, 1280
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    y = ops.gemm(x, w, b, splits=splits)
    r = x.float() @ w.float().t() + b.float()
    assert _rel_err(y, r) < 1e-2
    assert _tile_max_err(y, r) < 3e-2


def test_gemm_deterministic():
    torch.manual_seed(2)
    x = torch.randn(64, 2304, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(4096, 2304, device="cuda", dtype=torch.bfloat16)
    a = ops.gemm(x, w)
    b = ops.gemm(x, w)
    assert torch.equal(a, b)


@pytest.mark.parametrize("T,H", [(1, 2304), (77, 4096), (128, 512)])
def test_rms_norm(T, H):
    torch.manual_seed(0)
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    y = ops.rms_norm(x, w, 1e-6)
    r = ref.rms_norm(x.float(), w.float(), 1e-6)
    assert _rel_err(y, r) < 1e-2


def test_rms_norm_strided_rows():
    x = torch.randn(9, 576, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(512, device="cuda", dtype=torch.bfloat16)
    y = ops.rms_norm(x[:, :512], w, 1e-6)
    r = ref.rms_norm(x[:, :512].float(), w.float(), 1e-6)
    assert _rel_err(y, r) < 1e-2


def test_fused_add_rms_norm():
    torch.manual_seed(0)
    x = torch.randn(17, 2304, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(17, 2304, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2304, device="cuda", dtype=torch.bfloat16)
    x2, r2 = x.clone().cpu(), res.clone().cpu()
    ref.fused_add_rms_norm(x2, r2, w.cpu(), 1e-6)
    ops.fused_add_rms_norm(x, res, w, 1e-6)
    assert torch.equal(res.cpu(), r2)
    assert _rel_err(x.cpu(), x2) < 1e-2
