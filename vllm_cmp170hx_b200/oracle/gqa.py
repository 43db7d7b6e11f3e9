"""Gated grouped-query attention (the full-attention layers of the Qwen3-Next-style hybrid), fp32 math.

Per query head the projection gives [q | gate] (head_dim 256 each), then the key and value heads:

* ``q' = rope(bf16(rmsnorm(q) * w_q))`` and ``k' = rope(bf16(rmsnorm(k) * w_k))`` -- per-head RMSNorm, the
  normalised value rounded to bf16 (the projection's precision), NeoX RoPE on the first ``rot_dim`` dims;
* ``o = softmax(q' k'^T / sqrt(256)) v`` over the token's causal prefix of its sequence, query head h
  reading key-value head ``h // (nh / nkv)``;
* ``y = o * sigmoid(gate)`` (the attention output gate), then the row-parallel ``o_proj``.

These are the definitions the CUDA path (csrc/gqa.cu and the dense mode of the block attention kernel)
is tested against.
"""

from __future__ import annotations

import torch

from .mla import rope

HD = 256


def norm_rope(x: torch.Tensor, w: torch.Tensor, eps: float, positions: torch.Tensor,
              cos_sin: torch.Tensor) -> torch.Tensor:
    """x [T, heads, 256] -> rounded, rotated bf16 rows."""
    xf = x.float()
    y = xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps) * w.float()
    y = y.to(torch.bfloat16)
    return rope(y, positions, cos_sin, 0, cos_sin.shape[1], False).to(torch.bfloat16)


def split_proj(proj: torch.Tensor, nh: int, nkv: int):
    """proj [T, nh*512 + nkv*512] -> q [T, nh, 256], gate [T, nh, 256], k, v [T, nkv, 256]."""
    T = proj.shape[0]
    qg = proj[:, :nh * 2 * HD].reshape(T, nh, 2, HD)
    k = proj[:, nh * 2 * HD: nh * 2 * HD + nkv * HD].reshape(T, nkv, HD)
    v = proj[:, nh * 2 * HD + nkv * HD: nh * 2 * HD + 2 * nkv * HD].reshape(T, nkv, HD)
    return qg[:, :, 0], qg[:, :, 1], k, v


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """q [group, 256] of one token and key-value head; k, v [L, 256] its visible rows -> [group, 256] fp32."""
    s = (q.float() @ k.float().t()) * scale
    p = torch.softmax(s, dim=-1)
    return p @ v.float()


def layer_core(proj: torch.Tensor, nh: int, nkv: int, q_norm_w, k_norm_w, eps: float, positions: torch.Tensor,
               cos_sin: torch.Tensor, seq_starts: list[int], seq_lens: list[int]) -> torch.Tensor:
    """Whole prompts (no cache): proj [T, ...] of sequences laid out one after another (starts /
    lengths), positions from 0.  Returns y = o * sigmoid(gate) [T, nh*256] fp32."""
    q, gate, k, v = split_proj(proj, nh, nkv)
    qr = norm_rope(q, q_norm_w, eps, positions, cos_sin)
    kr = norm_rope(k, k_norm_w, eps, positions, cos_sin)
    G = nh // nkv
    T = proj.shape[0]
    y = torch.zeros(T, nh, HD)
    for a, n in zip(seq_starts, seq_lens):
        for i in range(n):
            t = a + i
            for j in range(nkv):
                o = attend(qr[t, j * G:(j + 1) * G], kr[a:t + 1, j], v[a:t + 1, j], HD ** -0.5)
                y[t, j * G:(j + 1) * G] = o.to(torch.bfloat16).float()
    return (y * torch.sigmoid(gate.float())).reshape(T, nh * HD)
