"""References of the dense building blocks: GEMM, RMSNorm, RoPE, activations."""

from __future__ import annotations

import torch


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w^T (+ bias) computed in fp32, returned in x's dtype."""
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(x.dtype)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """In place: residual = x + residual (rounded to its dtype); x = rms_norm(residual)."""
    r = (x.float() + residual.float()).to(residual.dtype)
    residual.copy_(r)
    x.copy_(rms_norm(r, w, eps))


def silu_and_mul(x: torch.Tensor, limit: float | None = None) -> torch.Tensor:
    """SwiGLU over the last dim split in halves [gate | up]; optional clamp as
    in csrc/exl3/common.h:77-98 of the reference (gate <= L, |up| <= L)."""
    d = x.shape[-1] // 2
    g, u = x[..., :d].float(), x[..., d:].float()
    if limit is not None:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return (torch.nn.functional.silu(g) * u).to(x.dtype)


def rope_neox(x: torch.Tensor, positions: torch.Tensor, base: float, rot_dim: int | None = None) -> torch.Tensor:
    """Rotary embedding, GPT-NeoX (half-split) style, on the first rot_dim dims of the last axis.
    x: [T, ..., D], positions: [T]."""
    D = x.shape[-1]
    rd = rot_dim or D
    half = rd // 2
    inv = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float64) / half))
    ang = positions.double()[:, None] * inv[None, :]
    cos, sin = ang.cos().float(), ang.sin().float()
    shape = [x.shape[0]] + [1] * (x.dim() - 2) + [half]
    cos, sin = cos.view(shape).to(x.device), sin.view(shape).to(x.device)
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:rd]
    out = xf.clone()
    out[..., :half] = x1 * cos - x2 * sin
    out[..., half:rd] = x2 * cos + x1 * sin
    return out.to(x.dtype)
