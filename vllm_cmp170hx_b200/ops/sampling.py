"""Greedy / temperature sampling over (vocab-sharded) logits."""

from __future__ import annotations

import torch

from .. import _ext


MAX_BANS = 4


def sample_local(logits: torch.Tensor, temperature: torch.Tensor | None, seed: int, step: torch.Tensor | None,
                 vocab_offset: int = 0, bans: torch.Tensor | None = None):
    """Per-row winner of this vocab shard: (value [rows] fp32, global index [rows] int32).
    Greedy rows (temperature <= 0) take the argmax; others the Gumbel-max sample.  bans [rows, <= 4]
    int32 global token ids that never win (-1 = none)."""
    rows = logits.shape[0]
    if not logits.is_cuda:
        # as the kernel: NaN never wins; a row without any finite winner reports index 2^31 - 1
        x = torch.nan_to_num(logits.float(), nan=float("-inf"))
        if bans is not None:
            V = x.shape[1]
            for r in range(rows):
                for t in bans[r].tolist():
                    if 0 <= t - vocab_offset < V:
                        x[r, t - vocab_offset] = float("-inf")
        if temperature is not None:
            g = torch.Generator().manual_seed(int(seed) + int(step.item() if step is not None else 0))
            u = torch.rand(x.shape, generator=g).clamp_(1e-12, 1 - 1e-7)
            t = temperature.float()[:, None]
            noisy = x / t.clamp_min(1e-6) - torch.log(-torch.log(u))
            x = torch.where(t > 0, noisy, x)
        v, i = x.max(dim=-1)  # torch.max returns the first maximal index
        i = torch.where(torch.isneginf(v), torch.full_like(i, 2**31 - 1 - vocab_offset), i)
        return v, (i + vocab_offset).int()
    val = torch.empty(rows, dtype=torch.float32, device=logits.device)
    idx = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _ext.ops().sample_rows(logits, temperature, int(seed), step, vocab_offset, val, idx, bans)
    return val, idx


def combine(vals: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """vals/idx [R, rows] per-shard winners -> token ids [rows] int64."""
    if not vals.is_cuda:
        best = vals.max(dim=0).values
        out = torch.empty(vals.shape[1], dtype=torch.int64)
        for r in range(vals.shape[1]):
            cand = idx[:, r][vals[:, r] == best[r]]
            out[r] = int(cand.min())
        return out
    out = torch.empty(vals.shape[1], dtype=torch.int64, device=vals.device)
    _ext.ops().sample_combine(vals.contiguous(), idx.contiguous(), out)
    return out
