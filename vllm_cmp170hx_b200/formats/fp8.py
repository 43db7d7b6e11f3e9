"""fp8 (e4m3) weights with one fp32 scale per 128 x 128 block (the DeepSeek
checkpoint convention: ``weight`` [N, K] e4m3 and ``weight_scale_inv``
[ceil(N/128), ceil(K/128)] fp32; value = q * s)."""

from __future__ import annotations

import torch

FP8_MAX = 448.0


def quantize(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32)
    wp[:N, :K] = w.float()
    blocks = wp.view(nb, block, kb, block)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / FP8_MAX
    q = (blocks / s[:, None, :, None]).to(torch.float8_e4m3fn).view(nb * block, kb * block)[:N, :K]
    return q.contiguous(), s.float()


def dequantize(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    full = s.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * full


def random_weight(N: int, K: int, std: float, generator=None, device="cpu"):
    w = torch.randn(N, K, generator=generator) * std
    q, s = quantize(w)
    return q.to(device), s.to(device)
