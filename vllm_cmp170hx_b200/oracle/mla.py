"""References of the sparse-MLA path (fp32 math).

Contracts follow the reference's DeepSeek-style sparse attention
(vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py:17-33):
indexer score(s) = sum_h w_h * relu(q_h . k_s); top-k among visible
positions, ties to the lowest position, selection ascending; attention over
the selected latent rows with q = [q_nope absorbed into the latent | q_rope].
"""

from __future__ import annotations

import math

import torch

from ..formats.exl3 import hadamard128

FP8_MAX = 448.0


def rope_cos_sin(max_pos: int, rot_dim: int, base: float = 10000.0, device="cpu") -> torch.Tensor:
    """[max_pos, rot_dim] fp32 table: cos of the rot_dim/2 frequencies, then sin."""
    half = rot_dim // 2
    inv = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float64) * 2 / rot_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).float().to(device)


def rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, offset: int, rot_dim: int,
         interleaved: bool) -> torch.Tensor:
    """x [T, H, D]; returns a rotated copy (fp32 math, x's dtype)."""
    half = rot_dim // 2
    cs = cos_sin[positions.long()].float()  # [T, rot_dim]
    c, s = cs[:, None, :half], cs[:, None, half:]
    y = x.float().clone()
    seg = y[..., offset:offset + rot_dim]
    if interleaved:
        a, b = seg[..., 0::2].clone(), seg[..., 1::2].clone()
        seg[..., 0::2] = a * c - b * s
        seg[..., 1::2] = b * c + a * s
    else:
        a, b = seg[..., :half].clone(), seg[..., half:].clone()
        seg[..., :half] = a * c - b * s
        seg[..., half:] = b * c + a * s
    return y.to(x.dtype)


def latent_row(kv: torch.Tensor, norm_w, eps, positions, cos_sin, interleaved) -> torch.Tensor:
    """[T, 576] bf16 cache rows: RMSNorm(kv[:, :512]) * w | RoPE(kv[:, 512:])."""
    c = kv[:, :512].float()
    c = c * torch.rsqrt((c * c).mean(-1, keepdim=True) + eps) * norm_w.float()
    pe = rope(kv[:, None, 512:576], positions, cos_sin, 0, 64, interleaved)[:, 0]
    return torch.cat([c.to(torch.bfloat16), pe.to(torch.bfloat16)], dim=1)


def quant_fp8(v: torch.Tensor):
    """Per-row e4m3 quantisation with scale amax/448: returns (q fp8, scale fp32)."""
    amax = v.abs().amax(-1, keepdim=True)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    return (v / scale).to(torch.float8_e4m3fn), scale[..., 0]


def index_k(k, ln_w, ln_b, eps, positions, cos_sin, interleaved):
    kf = k.float()
    mu = kf.mean(-1, keepdim=True)
    var = ((kf - mu) ** 2).mean(-1, keepdim=True)
    y = (kf - mu) * torch.rsqrt(var + eps)
    if ln_w is not None:
        y = y * ln_w.float()
    if ln_b is not None:
        y = y + ln_b.float()
    y = y.to(torch.bfloat16).float()
    y = rope(y[:, None], positions, cos_sin, 0, cos_sin.shape[1], interleaved)[:, 0].float()
    return hadamard128(y)


def index_q(q, positions, cos_sin, interleaved):
    y = rope(q.float(), positions, cos_sin, 0, cos_sin.shape[1], interleaved).float()
    return hadamard128(y)


def indexer_scores(q: torch.Tensor, w: torch.Tensor, keys: torch.Tensor) -> torch.Tensor:
    """q [H, D], w [H], keys [S, D] (all fp32) -> [S]."""
    return (torch.relu(keys @ q.t()) * w[None, :]).sum(-1)


def topk_positions(scores: torch.Tensor, ctx: int, k: int) -> torch.Tensor:
    """Ascending positions of the k largest of scores[:ctx] (ties: lowest position)."""
    if ctx <= k:
        return torch.arange(ctx)
    s = scores[:ctx]
    order = torch.argsort(-s, stable=True)[:k]
    return torch.sort(order).values


def sparse_attention(q: torch.Tensor, rows: torch.Tensor, sm_scale: float):
    """q [H, 576], rows [S, 576] (selected cache rows) -> (o [H, 512], lse [H])."""
    logits = (q.float() @ rows.float().t()) * sm_scale
    lse = torch.logsumexp(logits, dim=-1)
    p = torch.softmax(logits, dim=-1)
    return p @ rows[:, :512].float(), lse


def softmax_scale(qk_head_dim: int, mscale: float = 1.0) -> float:
    return mscale * mscale / math.sqrt(qk_head_dim)
