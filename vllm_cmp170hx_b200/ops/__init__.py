"""Python entry points of the sm_100a kernels.

Each function takes CUDA tensors to the native kernel (``torch.ops.b200.*``,
built from ``csrc/``) and CPU tensors to the plain-PyTorch oracle of the same
op (``vllm_cmp170hx_b200.oracle``), which is how the engine runs in CPU tests.
There is no third path: a CUDA tensor never falls back to eager PyTorch, and a
missing extension raises on first use.
"""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import basic as _ref


def _native(t: torch.Tensor) -> bool:
    return t.is_cuda


def gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
         splits: int = 0, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """y = x @ w^T (+ bias), bf16 inputs, fp32 accumulate, bf16 or fp32 output (tcgen05 on GPU)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if not _native(x2):
        y = (x2.float() @ w.float().t() + (bias.float() if bias is not None else 0)).to(out_dtype)
        if out is not None:
            out.view(-1, w.shape[0]).copy_(y)
            return out
        return y.view(*lead, w.shape[0])
    if x2.stride(-1) != 1 or (x2.stride(0) % 8 and x2.shape[0] > 1):
        x2 = x2.contiguous()  # TMA needs 16-byte row strides
    if out is None:
        out = torch.empty(*lead, w.shape[0], dtype=out_dtype, device=x.device)
    o2 = out.view(-1, w.shape[0])
    from ..parallel import sp as _sp

    spa = _sp.active()
    if spa is not None and spa.fused and spa.take_pending(x2):
        # x is the all-gather area of the sequence-parallel layout: the GEMM waits for it itself
        if bias is not None:
            raise ValueError("the all-gather GEMM takes no bias")
        spa.gemm_ag(x2, w, o2)
        return out
    if splits == 0:
        from .. import envs

        splits = envs.get("VLLM_B200_GEMM_SPLITK")
    _ext.ops().gemm_bf16_out(x2, w, bias, o2, _ext.status_word(x.device), splits)
    return out


def bmm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[b] = x[b] @ w[b]^T for x [B, M, K], w [B, N, K] (bf16, fp32 accumulate; any strides with a unit
    inner one, e.g. per-head slices of a [T, H, D] tensor transposed to [H, T, D])."""
    if out is None:
        out = torch.empty(x.shape[0], x.shape[1], w.shape[1], dtype=torch.bfloat16, device=x.device)
    if not _native(x):
        out.copy_(torch.bmm(x.float(), w.float().transpose(1, 2)).to(out.dtype))
        return out
    _ext.ops().gemm_batched(x, w, out, _ext.status_word(x.device))
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if not _native(x):
        y = _ref.rms_norm(x2, w, eps)
        if out is not None:
            out.reshape(-1, x.shape[-1]).copy_(y)
            return out
        return y.view(*lead, x.shape[-1])
    if out is None:
        out = torch.empty(*lead, x.shape[-1], dtype=x.dtype, device=x.device)
    _ext.ops().rms_norm_out(out.view(-1, x.shape[-1]) if out.dim() != 2 else out, x2, w, eps)
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """In place: residual += x; x = rms_norm(residual) * w."""
    if not _native(x):
        _ref.fused_add_rms_norm(x, residual, w, eps)
        return
    _ext.ops().fused_add_rms_norm(x, residual, w, eps)


def silu_mul(x: torch.Tensor, limit: float = 0.0, out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU of [gate | up] halves of the last dim (optional clamp)."""
    I = x.shape[-1] // 2
    if not _native(x):
        y = _ref.silu_and_mul(x, limit or None)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(*x.shape[:-1], I, dtype=x.dtype, device=x.device)
    _ext.ops().silu_mul(out.view(-1, I), x.view(-1, 2 * I), float(limit))
    return out
