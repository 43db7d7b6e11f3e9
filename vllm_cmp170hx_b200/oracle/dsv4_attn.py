"""fp32 definition of the DeepSeek-V4.1 attention core, per token.

For a query at absolute position p the attended rows are

* the window: the layer's rows of positions [max(0, p - window + 1), p], each RoPE'd at its
  position and then FP8 (blocks of 32, power-of-two scales) quantize-dequantized;
* the compressed rows: n_vis = (p + 1) // ratio groups of `ratio` consecutive positions are closed;
  group g's row is the RMS-normalised latent of the group (ratio 1: the token's own row; ratio 2:
  the pair pooled by an fp32 softmax over its gate scores), RoPE'd at the group's first position
  and FP4 (blocks of 16, E4M3 scales) quantize-dequantized.  When n_vis exceeds the indexer's
  top-k only the top-k best groups are attended.

The indexer scores group g for the query as sum over index heads of
bf16(bf16(relu(bf16(q_h . k_g))) * w_h), the heads summed in fp32 per tensor-parallel rank group and
rounded to bf16, the groups added in rank order (the all-reduce); index keys are
FP4(RoPE(RMSNorm(wk(latent)))) with power-of-two scales per 32, the index query likewise.  The
selection is canonical (score descending, position ascending on ties, then sorted ascending).  A
second level may restrict the choice to candidate blocks picked by another layer's indexer (the
block holding the newest visible group always in); visible groups outside them score -FLT_MAX.

Attention is MQA over rows that serve as both K and V (512 dims, RoPE on the last 64): fp32 scores
times head_dim^-0.5, softmax whose denominator also holds exp(sink_h), probabilities rounded to bf16
before they weight the rows; a query with no row gets zeros.  The output gets the inverse RoPE on
its tail and an FP8 quantize-dequantize per output group (the wo_a input).

This is an independent statement of the math the reference implements in
vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py (window_kv :262, compress_rows :294,
index_key_rows :371, compressed_kv :384, index_query :433, combine_head_scores :450,
topk_canonical :523, select_candidate_blocks :569, mask_to_candidates :598, sparse_attention_torch
:678, output_qdq :736) and its quantize-dequantize definitions (ops/sm80_act_quant.py:1-32).
"""

from __future__ import annotations

import torch

FLT_MAX = torch.finfo(torch.float32).max
_FP8_MAX = 448.0
_FP4_MAX = 6.0
_INV_FP8 = float(torch.tensor(1.0 / 448.0, dtype=torch.float32))
_INV_FP4 = float(torch.tensor(1.0 / 6.0, dtype=torch.float32))


# ---------------------------------------------------------------------------- quantize-dequantize
def _pow2_at_least(a: torch.Tensor) -> torch.Tensor:
    """The smallest power of two >= a, for positive normal fp32 a (from its exponent bits)."""
    b = a.float().contiguous().view(torch.int32)
    e = ((b >> 23) & 0xFF) + ((b & 0x7FFFFF) != 0).to(torch.int32)
    return (e << 23).view(torch.float32)


def _round_e2m1(v: torch.Tensor) -> torch.Tensor:
    """fp32 onto {0, .5, 1, 1.5, 2, 3, 4, 6} (signed), nearest with ties to even; |v| <= 6."""
    a = v.abs()
    step = torch.where(a < 2, 0.5, torch.where(a < 4, 1.0, 2.0))
    return torch.copysign(torch.round(a / step) * step, v)


def _round_e4m3(v: torch.Tensor) -> torch.Tensor:
    return v.clamp(-_FP8_MAX, _FP8_MAX).to(torch.float8_e4m3fn).float()


def qdq_fp8(x: torch.Tensor, block: int = 32) -> torch.Tensor:
    """Per `block` values of the last dim: s = pow2 >= max(absmax, 1e-4) / 448, y = e4m3(x / s) s."""
    shp = x.shape
    b = x.float().reshape(*shp[:-1], shp[-1] // block, block)
    s = _pow2_at_least(b.abs().amax(-1, keepdim=True).clamp_min(1e-4) * _INV_FP8)
    return (_round_e4m3(b / s) * s).reshape(shp).to(x.dtype)


def qdq_fp4(x: torch.Tensor, block: int, scale: str = "e8m0") -> torch.Tensor:
    """Per `block` values: e8m0 s = pow2 >= max(absmax, 6 * 2^-126) / 6; e4m3 s = e4m3(max(absmax,
    6 * 2^-9) / 6) (saturating); y = e2m1(clamp(x / s, -6, 6)) s."""
    shp = x.shape
    b = x.float().reshape(*shp[:-1], shp[-1] // block, block)
    amax = b.abs().amax(-1, keepdim=True)
    if scale == "e8m0":
        s = _pow2_at_least(amax.clamp_min(6 * 2.0 ** -126) * _INV_FP4)
    elif scale == "e4m3":
        s = _round_e4m3(amax.clamp_min(6 * 2.0 ** -9) / _FP4_MAX)
    else:
        raise ValueError(scale)
    return (_round_e2m1((b / s).clamp(-_FP4_MAX, _FP4_MAX)) * s).reshape(shp).to(x.dtype)


# ---------------------------------------------------------------------------- elementwise
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return (w.float() * xf).to(x.dtype)


def rope(x: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Rotate the last 2 len(freqs) dims of x [T, ..., D] (adjacent pairs as complex numbers) by
    position * freq (fp32 angles, complex64 product), one rounding to x's dtype."""
    rd = 2 * freqs.numel()
    ang = positions.float().unsqueeze(-1) * freqs.float()
    cis = torch.polar(torch.ones_like(ang), ang)
    if inverse:
        cis = cis.conj()
    cis = cis.view((positions.shape[0],) + (1,) * (x.dim() - 2) + (rd // 2,))
    tail = torch.view_as_complex(x[..., -rd:].float().reshape(*x.shape[:-1], rd // 2, 2).contiguous())
    out = x.clone()
    out[..., -rd:] = torch.view_as_real(tail * cis).flatten(-2).to(x.dtype)
    return out


# ---------------------------------------------------------------------------- KV rows
def window_rows(kv: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Cached window rows of kv [T, 512] (bf16, pre-RoPE)."""
    return qdq_fp8(rope(kv, positions, freqs), 32)


def pool_pair(prev: torch.Tensor, cur: torch.Tensor, norm_w: torch.Tensor, eps: float) -> torch.Tensor:
    """Ratio-2 group latent from the group's two fp32 [kv | score] rows [n, 2 d]."""
    d = prev.shape[-1] // 2
    kv = torch.stack((prev[..., :d], cur[..., :d]), -2)
    sc = torch.stack((prev[..., d:], cur[..., d:]), -2)
    pooled = (kv * sc.softmax(-2)).sum(-2)
    return rms_norm(pooled.to(torch.bfloat16), norm_w, eps)


def compressed_rows(latent: torch.Tensor, group_pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    return qdq_fp4(rope(latent, group_pos, freqs), 16, "e4m3")


def index_key_rows(k: torch.Tensor, k_norm: torch.Tensor, freqs: torch.Tensor, group_pos: torch.Tensor,
                   eps: float) -> torch.Tensor:
    return qdq_fp4(rope(rms_norm(k, k_norm, eps), group_pos, freqs), 32, "e8m0")


def index_query(q: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    return qdq_fp4(rope(q, positions, freqs), 32, "e8m0")


# ---------------------------------------------------------------------------- indexer
def index_scores(q: torch.Tensor, w: torch.Tensor, keys: torch.Tensor, n_vis: torch.Tensor,
                 heads_per_rank: int) -> torch.Tensor:
    """q [n, H, D] bf16, w [n, H] bf16, keys [N, D] -> [n, N] fp32 (bf16 values), -inf past n_vis."""
    return index_scores_rows(q, w, keys.unsqueeze(0).expand(q.shape[0], -1, -1), n_vis, heads_per_rank)


def index_scores_rows(q: torch.Tensor, w: torch.Tensor, keys: torch.Tensor, n_vis: torch.Tensor,
                      heads_per_rank: int) -> torch.Tensor:
    """index_scores with each query's own keys [n, N, D] (queries of different sequences)."""
    bf = torch.bfloat16
    s = torch.einsum("nhd,nkd->nhk", q.float(), keys.float()).to(bf).float().clamp_min(0)
    s = (s * w.float().unsqueeze(-1)).to(bf).float()
    total = None
    for r0 in range(0, s.shape[1], heads_per_rank):
        part = s[:, r0]
        for h in range(r0 + 1, r0 + heads_per_rank):
            part = part + s[:, h]
        part = part.to(bf).float()
        total = part if total is None else (total + part).to(bf).float()
    cols = torch.arange(keys.shape[1], device=q.device)
    return torch.where(cols[None] < n_vis[:, None], total, float("-inf"))


def topk_canonical(scores: torch.Tensor, n_vis: torch.Tensor, k: int) -> torch.Tensor:
    """min(k, n_vis) best columns per row (score desc, index asc), sorted ascending, -1 padded."""
    n, N = scores.shape
    dev = scores.device
    out = torch.full((n, k), -1, dtype=torch.int32, device=dev)
    w = min(k, N)
    if n == 0 or w == 0:
        return out
    cols = torch.arange(N, device=dev)
    sc = torch.where(cols[None] < n_vis[:, None], scores, float("-inf"))
    order = torch.sort(sc, dim=-1, descending=True, stable=True).indices[:, :w]
    keep = torch.arange(w, device=dev)[None] < n_vis[:, None]
    picked = torch.sort(torch.where(keep, order, N), -1).values
    out[:, :w] = torch.where(picked == N, -1, picked).to(torch.int32)
    return out


def candidate_blocks(scores: torch.Tensor, n_vis: torch.Tensor, topk_blocks: int, block: int) -> torch.Tensor:
    """Blocks of `block` groups scored by their best group; the block of the newest visible group
    pinned in; the best `topk_blocks` reachable blocks, sorted ascending, -1 padded."""
    n, N = scores.shape
    pad = -N % block
    b = torch.nn.functional.pad(scores, (0, pad), value=float("-inf")).reshape(n, -1, block).amax(-1)
    nb = b.shape[1]
    last = torch.div(n_vis - 1, block, rounding_mode="floor")
    b = b.masked_fill(torch.arange(nb, device=scores.device)[None] == last[:, None], float("inf"))
    out = torch.full((n, topk_blocks), -1, dtype=torch.int32, device=scores.device)
    w = min(topk_blocks, nb)
    if n == 0 or w == 0:
        return out
    top = torch.sort(b, dim=-1, descending=True, stable=True)
    ids = torch.where(top.values[:, :w] > float("-inf"), top.indices[:, :w], nb)
    ids = torch.sort(ids, -1).values
    out[:, :w] = torch.where(ids == nb, -1, ids).to(torch.int32)
    return out


def mask_to_candidates(scores: torch.Tensor, cands: torch.Tensor, block: int) -> torch.Tensor:
    n, N = scores.shape
    nb = -(-N // block)
    keep = torch.zeros(n, nb + 1, dtype=torch.bool, device=scores.device)
    ids = torch.where((cands >= 0) & (cands < nb), cands, nb).long()
    keep.scatter_(1, ids, True)
    keep = keep[:, :nb].repeat_interleave(block, 1)[:, :N]
    return torch.where(keep | (scores == float("-inf")), scores, -FLT_MAX)


# ---------------------------------------------------------------------------- attention
def sparse_attention(q: torch.Tensor, rows: torch.Tensor, valid: torch.Tensor, sink: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """q [n, h, d], rows [n, R, d] (K = V), valid [n, R] -> [n, h, d] bf16."""
    s = torch.einsum("nhd,nrd->nhr", q.float(), rows.float()) * scale
    s = s.masked_fill(~valid[:, None, :], float("-inf"))
    m = s.amax(-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.full_like(m, -1e30))
    p = torch.exp(s - m)
    den = p.sum(-1) + torch.exp(sink[None, :].float() - m.squeeze(-1))
    o = torch.einsum("nhr,nrd->nhd", p.to(torch.bfloat16).float(), rows.float())
    return (o / den.unsqueeze(-1)).to(torch.bfloat16)


def output_qdq(o: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, n_groups: int) -> torch.Tensor:
    n, h, d = o.shape
    o = rope(o, positions, freqs, inverse=True)
    return qdq_fp8(o.reshape(n, n_groups, (h // n_groups) * d), 32).reshape(n, h, d)
