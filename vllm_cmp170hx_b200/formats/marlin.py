"""Marlin-packed uint4b8 group-128 weights (vLLM's Marlin MoE layout, the one
the reference's decode kernels read, csrc/ampere_marlin/decode_v2.cu:15-23).

* packed int32 ``[K/16, 2N]`` per matrix (``[E, K/16, 2N]`` for experts): for
  k16 row r, 64-column tile t, lane l and int32 j, the word sits at
  ``(t*32 + l)*4 + j`` of row r; with c = l % 4, g = l // 4 its nibbles hold
  (k, n) = nib0 (2c, g), nib1 (2c+8, g), nib2 (2c, g+8), nib3 (2c+8, g+8),
  nib4 (2c+1, g), nib5 (2c+9, g), nib6 (2c+1, g+8), nib7 (2c+9, g+8), with n
  relative to 64t + 16j.  Value = (q - 8) * s.
* scales bf16 ``[K/128, N]``: inside each 64-column chunk, column c is stored
  at position 8*(c % 8) + c // 8.
These positions are the format's; a reader of the format has no choice.
"""

from __future__ import annotations

import torch

# (dk, dn) of nibble i relative to (2c, g)
NIB = [(0, 0), (8, 0), (0, 8), (8, 8), (1, 0), (9, 0), (1, 8), (9, 8)]


def _index_maps(K: int, N: int):
    """For every packed (row, word, nibble): the (k, n) it holds."""
    r = torch.arange(K // 16).view(-1, 1, 1, 1, 1)
    t = torch.arange(N // 64).view(1, -1, 1, 1, 1)
    l = torch.arange(32).view(1, 1, -1, 1, 1)
    j = torch.arange(4).view(1, 1, 1, -1, 1)
    nib = torch.arange(8).view(1, 1, 1, 1, -1)
    dk = torch.tensor([d[0] for d in NIB])[nib]
    dn = torch.tensor([d[1] for d in NIB])[nib]
    c, g = l % 4, l // 4
    k = r * 16 + 2 * c + dk
    n = t * 64 + 16 * j + g + dn
    return k.expand(K // 16, N // 64, 32, 4, 8), n.expand(K // 16, N // 64, 32, 4, 8)


def scale_perm(N: int) -> torch.Tensor:
    """stored position -> logical column, per row of scales."""
    c = torch.arange(N)
    chunk, cc = c // 64, c % 64
    pos = chunk * 64 + 8 * (cc % 8) + cc // 8
    inv = torch.empty(N, dtype=torch.long)
    inv[pos] = c
    return inv


def pack(q: torch.Tensor, scales: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """q uint4 values [K, N] (0..15), scales [K/128, N] -> (packed int32 [K/16, 2N], stored scales)."""
    K, N = q.shape
    k, n = _index_maps(K, N)
    nibs = q[k, n].to(torch.int64)  # [K/16, N/64, 32, 4, 8]
    words = torch.zeros(nibs.shape[:-1], dtype=torch.int64)
    for i in range(8):
        words |= (nibs[..., i] & 15) << (4 * i)
    words = torch.where(words >= 1 << 31, words - (1 << 32), words).to(torch.int32)
    packed = words.reshape(K // 16, 2 * N)
    stored = torch.empty_like(scales)
    stored[:, :] = scales[:, scale_perm(N)]
    return packed, stored


def unpack(packed: torch.Tensor, stored_scales: torch.Tensor) -> torch.Tensor:
    """Dense bf16 weight [K, N] = bf16((q - 8) * s)."""
    K, N = packed.shape[0] * 16, packed.shape[1] // 2
    k, n = _index_maps(K, N)
    words = packed.reshape(K // 16, N // 64, 32, 4).to(torch.int64) & 0xFFFFFFFF
    q = torch.zeros(K, N, dtype=torch.int64)
    for i in range(8):
        q[k[..., i], n[..., i]] = (words >> (4 * i)) & 15
    s = torch.empty_like(stored_scales)
    s[:, scale_perm(N)] = stored_scales
    return ((q - 8).to(torch.float32) * s.float().repeat_interleave(128, dim=0)).to(torch.bfloat16)


def random_experts(E: int, K: int, N: int, generator=None, device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """Random packed weights (every int32 is a valid code) and positive scales ~ 1/(4 sqrt(K))."""
    g = generator
    packed = torch.randint(-(1 << 31), 1 << 31, (E, K // 16, 2 * N), dtype=torch.int64, generator=g).to(torch.int32)
    scales = (torch.rand(E, K // 128, N, generator=g) * 0.5 + 0.75) * (0.25 / K ** 0.5)
    return packed.to(device), scales.to(torch.bfloat16).to(device)
