"""Gated grouped-query attention ops: CUDA tensors run the kernels of csrc/gqa.cu and the dense mode of
the block attention kernel (csrc/mla_attn.cu); CPU tensors run the fp32 definitions of oracle/gqa.py.

Cache layout: one 512-wide bf16 row per (position, key-value head), ``[k' | v]``, at row
``slot * nkv + head`` (slot = block * 64 + offset, block size 64, as the other paged caches).  Query
rows are ``[T * nkv, group, 512]`` = ``[q' | 0]``, grouped by key-value head, so one attention CTA
serves a key-value head's query heads; the attention writes the value half of its output rows.
"""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import gqa as _ref

HD = _ref.HD


def prep(proj: torch.Tensor, nh: int, nkv: int, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, eps: float,
         positions: torch.Tensor, cos_sin: torch.Tensor, slots: torch.Tensor, q_out: torch.Tensor,
         cache: torch.Tensor) -> None:
    """Normalise + rotate the step's q into q_out [T*nkv, group, 512] and write [k' | v] of every token
    with slot >= 0 into the cache."""
    if proj.is_cuda:
        _ext.ops().gqa_prep(proj, nh, nkv, q_norm_w, k_norm_w, eps, positions, cos_sin, slots, q_out, cache)
        return
    T = proj.shape[0]
    q, _, k, v = _ref.split_proj(proj, nh, nkv)
    G = nh // nkv
    qr = _ref.norm_rope(q, q_norm_w, eps, positions, cos_sin)  # [T, nh, 256]
    qo = q_out.view(T, nkv, G, 2 * HD)
    qo[..., :HD] = qr.view(T, nkv, G, HD)
    qo[..., HD:] = 0
    kr = _ref.norm_rope(k, k_norm_w, eps, positions, cos_sin)
    keep = slots >= 0
    rows = cache.view(-1, nkv, 2 * HD)
    sl = slots[keep].long()
    rows[sl, :, :HD] = kr[keep]
    rows[sl, :, HD:] = v[keep].to(cache.dtype)


def pick_splits(Tq: int, max_ctx: int, num_sms: int = 148) -> int:
    """Position splits of the dense attention: enough CTAs for about two waves when there are few query
    rows, never more than the 128-position blocks of the longest context (at most 16)."""
    blocks = max(1, (max_ctx + 127) // 128)
    want = max(1, -(-2 * num_sms // max(Tq, 1)))
    return max(1, min(want, blocks, 16))


def attention(q: torch.Tensor, cache: torch.Tensor, ctx_lens: torch.Tensor, token_seq: torch.Tensor,
              block_table: torch.Tensor, nkv: int, max_ctx: int, out: torch.Tensor | None = None,
              splits: int | None = None) -> torch.Tensor:
    """Causal attention of q [T*nkv, group, 512] over the paged rows: returns [T*nkv, group, 512] whose
    value half [256, 512) holds o (bf16)."""
    Tq, G, _ = q.shape
    if out is None:
        out = torch.empty(Tq, G, 2 * HD, dtype=torch.bfloat16, device=q.device)
    if q.is_cuda:
        s = splits if splits is not None else pick_splits(Tq, max_ctx)
        _ext.ops().gqa_attention(q, cache, ctx_lens, token_seq, block_table, nkv, HD ** -0.5, s, out,
                                 _ext.status_word(q.device))
        return out
    rows = cache.view(-1, nkv, 2 * HD)
    T = Tq // nkv
    for t in range(T):
        L = int(ctx_lens[t])
        bt = block_table[int(token_seq[t])].long()
        pos = torch.arange(L)
        sl = bt[pos // 64] * 64 + pos % 64
        for j in range(nkv):
            r = rows[sl, j]
            o = _ref.attend(q[t * nkv + j, :, :HD], r[:, :HD], r[:, HD:], HD ** -0.5)
            out[t * nkv + j, :, HD:] = o.to(out.dtype)
    return out


def gate(attn: torch.Tensor, proj: torch.Tensor, nh: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [T, nh*256] = o * sigmoid(gate) from the attention rows and the projection's gate halves."""
    T = proj.shape[0]
    if out is None:
        out = torch.empty(T, nh * HD, dtype=torch.bfloat16, device=proj.device)
    if proj.is_cuda:
        _ext.ops().gqa_gate(attn, proj, nh, out)
        return out
    o = attn.view(T, nh, 2 * HD)[..., HD:].float()
    g = proj[:, :nh * 2 * HD].reshape(T, nh, 2, HD)[:, :, 1].float()
    out.copy_((o * torch.sigmoid(g)).reshape(T, nh * HD).to(out.dtype))
    return out
