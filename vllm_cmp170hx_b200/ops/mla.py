"""Sparse-MLA ops: RoPE, cache writes, indexer, top-k, latent attention."""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import mla as _ref


def rope_(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, offset: int, rot_dim: int,
          interleaved: bool) -> torch.Tensor:
    """In-place RoPE on x [T, heads, dim] (dims offset..offset+rot_dim)."""
    if not x.is_cuda:
        x.copy_(_ref.rope(x, positions, cos_sin, offset, rot_dim, interleaved))
        return x
    _ext.ops().rope(x, positions, cos_sin, offset, rot_dim, interleaved)
    return x


def rope_into(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, offset: int, rot_dim: int,
              interleaved: bool, out: torch.Tensor, out_offset: int) -> torch.Tensor:
    """out[:, :, out_offset:out_offset + rot_dim] = RoPE of x[:, :, offset:offset + rot_dim] (one kernel:
    the MLA query's rope dims go straight next to its absorbed part)."""
    if not x.is_cuda:
        y = _ref.rope(x, positions, cos_sin, offset, rot_dim, interleaved)
        out[:, :, out_offset:out_offset + rot_dim] = y[:, :, offset:offset + rot_dim]
        return out
    _ext.ops().rope(x, positions, cos_sin, offset, rot_dim, interleaved, out, out_offset)
    return out


def latent_cache_write(kv, norm_w, eps, positions, cos_sin, interleaved, slots, cache):
    if not kv.is_cuda:
        rows = _ref.latent_row(kv, norm_w, eps, positions, cos_sin, interleaved)
        ok = slots >= 0
        cache[slots[ok]] = rows[ok]
        return
    _ext.ops().mla_latent_cache_write(kv, norm_w, eps, positions, cos_sin, interleaved, slots, cache)


def index_k_write(k, ln_w, ln_b, eps, positions, cos_sin, interleaved, slots, cache, cache_scale):
    if not k.is_cuda:
        y = _ref.index_k(k, ln_w, ln_b, eps, positions, cos_sin, interleaved)
        q, s = _ref.quant_fp8(y)
        ok = slots >= 0
        cache[slots[ok]] = q.view(torch.uint8)[ok]
        cache_scale[slots[ok]] = s[ok]
        return
    _ext.ops().mla_index_k_write(k, ln_w, ln_b, eps, positions, cos_sin, interleaved, slots, cache, cache_scale)


def index_q_prep(q, positions, cos_sin, interleaved, w, wscale):
    """q [T, H, 128] -> (q8 [T, H, 128] uint8 (e4m3 bits), w' [T, H] fp32 with the q scale folded in)."""
    T, H, _ = q.shape
    if not q.is_cuda:
        y = _ref.index_q(q, positions, cos_sin, interleaved)
        q8, s = _ref.quant_fp8(y)
        return q8.view(torch.uint8), w.float() * wscale * s
    q8 = torch.empty(T, H, 128, dtype=torch.uint8, device=q.device)
    wo = torch.empty(T, H, dtype=torch.float32, device=q.device)
    _ext.ops().mla_index_q_prep(q, positions, cos_sin, interleaved, w, wscale, q8, wo)
    return q8, wo


def indexer_topk(q8, w, k_cache, k_scale, ctx_lens, token_seq, block_table, block_size: int, topk: int, max_ctx: int,
                 scores_buf: torch.Tensor | None = None):
    """Indexer scores over each token's visible positions, then the canonical top-k.
    Returns (indices [T, topk] int32 cache rows, -1 padded; counts [T] int32)."""
    T = q8.shape[0]
    dev = q8.device
    if not q8.is_cuda:
        idx = torch.full((T, topk), -1, dtype=torch.int32)
        cnt = torch.zeros(T, dtype=torch.int32)
        qd = q8.view(torch.float8_e4m3fn).float()
        for t in range(T):
            s = int(token_seq[t]) if token_seq is not None else t
            c = int(ctx_lens[t])
            p = torch.arange(c)
            rows = block_table[s][p // block_size].long() * block_size + p % block_size
            keys = k_cache[rows].view(torch.float8_e4m3fn).float() * k_scale[rows][:, None]
            sc = _ref.indexer_scores(qd[t], w[t], keys)
            sel = _ref.topk_positions(sc, c, topk)
            idx[t, : len(sel)] = rows[sel].int()
            cnt[t] = len(sel)
        return idx, cnt
    ops = _ext.ops()
    if scores_buf is None or scores_buf.shape[0] < T or scores_buf.shape[1] < max_ctx:
        scores_buf = torch.empty(T, max(max_ctx, 1), dtype=torch.float32, device=dev)
    ops.mla_indexer_scores(q8, w, k_cache, k_scale, ctx_lens, token_seq, block_table, max_ctx, scores_buf,
                           _ext.status_word(dev))
    idx = torch.empty(T, topk, dtype=torch.int32, device=dev)
    cnt = torch.empty(T, dtype=torch.int32, device=dev)
    ops.mla_topk(scores_buf, ctx_lens, topk, token_seq, block_table, block_size, idx, cnt)
    return idx, cnt


def pick_splits(T: int, nh: int, topk: int = 2048, num_sms: int = 148, max_partial_bytes: int = 512 << 20,
                block_us: float = 2.0, merge_bytes_per_us: float = 5e6) -> int:
    """Position splits of the block attention kernel (blocks of 128 positions): the count with the
    least estimated time = waves x blocks per CTA x the time of one block on one SM, plus the merge
    pass over the fp32 partial outputs (written and read once) when split.  VLLM_B200_SPARSE_MLA_SPLITS
    forces the count."""
    from .. import envs

    forced = envs.get("VLLM_B200_SPARSE_MLA_SPLITS")
    if forced > 0:
        return min(forced, max(1, (topk + 127) // 128))
    from ..tuning_table import lookup

    base = T * ((nh + 127) // 128) * 2  # CTAs per split: tokens x head groups x latent halves
    nblk = max(1, min((topk + 127) // 128, lookup("sparse_mla", "max_splits", {}, 8)))
    best, best_cost = 1, None
    for s in range(1, nblk + 1):
        part = s * T * nh * 512 * 4
        if s > 1 and part > max_partial_bytes:
            break
        waves = -(-base * s // num_sms)
        cost = waves * -(-nblk // s) * block_us + ((2 * part) / merge_bytes_per_us if s > 1 else 0.0)
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def sparse_attention(q: torch.Tensor, cache: torch.Tensor, indices: torch.Tensor, counts: torch.Tensor,
                     sm_scale: float, splits: int | None = None, want_lse: bool = False, only_half: int = -1):
    """q [T, nh, 576] (absorbed nope | rope) -> o_lat [T, nh, 512] bf16 (and lse [T, nh]).  only_half 0 / 1:
    compute only that 256-wide half of the output (the other half is left unwritten)."""
    T, nh, _ = q.shape
    if not q.is_cuda:
        out = torch.zeros(T, nh, 512, dtype=torch.bfloat16)
        lse = torch.full((T, nh), float("-inf"))
        for t in range(T):
            c = int(counts[t])
            if c == 0:
                continue
            rows = cache[indices[t, :c].long()]
            o, l = _ref.sparse_attention(q[t], rows, sm_scale)
            out[t] = o.to(torch.bfloat16)
            lse[t] = l
        return (out, lse) if want_lse else out
    out = torch.empty(T, nh, 512, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(T, nh, dtype=torch.float32, device=q.device) if want_lse else None
    s = splits if splits is not None else pick_splits(T, nh, indices.shape[1])
    _ext.ops().mla_sparse_attention(q.contiguous(), cache, indices, counts, sm_scale, s, out, lse,
                                    _ext.status_word(q.device), None, only_half)
    return (out, lse) if want_lse else out
