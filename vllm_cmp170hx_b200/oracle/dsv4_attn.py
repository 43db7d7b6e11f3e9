"""Host definition of the DeepSeek-V4.1 attention core (the fp32 model of what the CUDA path computes).

The contract, stated for one query token at absolute position ``p`` of a sequence:

Rows it may attend (every row is 512 wide and serves as both key and value; the last 64 dims carry RoPE):

* window rows: the layer's ``kv`` rows of positions ``max(0, p - window + 1) .. p``, each rotated by its
  own position and then rounded onto the FP8 grid (E4M3 codes, one power-of-two scale per 32 values);
* compressed rows: once ``ratio`` consecutive positions are complete they form a group.  At ratio 1 a
  group is the RMS-normalised compressor row of its token; at ratio 2 the two tokens' fp32 compressor rows
  ``[kv | score]`` are pooled with weights softmax(score) (per channel) and the pooled row is rounded to
  bf16 and RMS-normalised.  The group row is rotated by the group's first position and rounded onto the
  FP4 grid (E2M1 codes, one E4M3 scale per 16 values).  ``(p + 1) // ratio`` groups are visible.

Indexer: index keys are FP4 (E2M1, power-of-two scale per 32) of the rotated, RMS-normalised
``wk(latent)``; the index query is likewise FP4 of the rotated query.  The score of group ``g`` is
built from per-head terms ``t_h = bf16(w_h * relu(bf16(q_h . k_g)))``; the heads of each tensor-parallel
rank group are added in head order in fp32 and the sum rounded to bf16, and the rank groups' sums are
added in rank order with a bf16 rounding after each addition (the all-reduce).  The chosen groups are
the ``min(topk, visible)`` best by (score descending, group ascending), listed in ascending group
order.  A second level may first restrict the candidates to blocks of ``block`` groups chosen by another
layer's indexer; groups outside those blocks then score -FLT_MAX (not -inf: they stay selectable when
too few candidates exist).  The blocks a source layer publishes are the ``topk_blocks`` best by their
best group's score (block of the newest visible group always in), ascending.

Attention: MQA with fp32 logits ``q . row * 512^-0.5``; softmax weights ``e_r = exp(l_r - max_r l_r)``
whose denominator also holds ``exp(sink_h - max_r l_r)``; the rows are weighted by the bf16-rounded
``e_r`` and divided by the fp32 denominator; a query without any row gets zeros.  The output's tail is
rotated back (inverse RoPE) and rounded onto the FP8 grid per 32 values (the input of ``wo_a``).

Grids and scales (blocks along the last dim):

* FP8: ``s = 2^ceil(log2(max(amax, 1e-4) * fl32(1/448)))``, ``y = e4m3(x / s) * s``;
* FP4 with power-of-two scales: ``s = 2^ceil(log2(max(amax, 6 * 2^-126) * fl32(1/6)))``;
* FP4 with E4M3 scales: ``s = e4m3(max(amax, 6 * 2^-9) / 6)``;
* FP4 values: ``e2m1(clamp(x / s, -6, 6)) * s`` with E2M1 rounding to nearest, ties to the even code.

The model these rounding points define is the reference's (vllm_sm80/models/deepseek_v41/ops/
sm80_attn_core.py: window rows :262, compressed rows :294-384, indexer :433-470, selection :523-610,
attention :678, output :736; FP8 / FP4 grids ops/sm80_act_quant.py:1-32).  The code below is written
from that statement: rotations in fp64 from fp32 angles, scales from ``frexp``, E2M1 by rounding
thresholds, and selections by one sortable 64-bit key per candidate.
"""

from __future__ import annotations

import torch

NEG_FLT_MAX = -torch.finfo(torch.float32).max
E4M3_MAX = 448.0
E2M1_MAX = 6.0
# the reciprocals the scale rules multiply by, as fp32 numbers
RECIP_E4M3_MAX = float(torch.tensor(1.0 / E4M3_MAX, dtype=torch.float32))
RECIP_E2M1_MAX = float(torch.tensor(1.0 / E2M1_MAX, dtype=torch.float32))


# ---------------------------------------------------------------------------- number grids
def pow2_ceil(a: torch.Tensor) -> torch.Tensor:
    """2^ceil(log2 a) for positive normal fp32 a: frexp gives a = m 2^e with m in [0.5, 1); a is itself
    a power of two exactly when m == 0.5."""
    m, e = torch.frexp(a.float())
    return torch.ldexp(torch.ones_like(m), e - (m == 0.5).to(e.dtype))


def e4m3(v: torch.Tensor) -> torch.Tensor:
    """Nearest E4M3 value (saturating at +-448), as fp32."""
    return v.float().clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()


# E2M1 magnitudes and the rounding thresholds between neighbours; a magnitude exactly on a threshold
# goes to the neighbour with the even code (0, 1, 2, 4 have even codes; 0.5, 1.5, 3, 6 odd)
_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1_THRESHOLDS = ((0.25, False), (0.75, True), (1.25, False), (1.75, True), (2.5, False), (3.5, True), (5.0, False))


def e2m1(v: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 value of v (|v| <= 6), ties to the even code, as fp32.  The magnitude is the sum of
    the steps between neighbouring grid values whose threshold v passes (no table tensor, so the
    function runs inside CUDA-graph capture)."""
    a = v.float().abs()
    mag = torch.zeros_like(a)
    for (t, tie_up), lo, hi in zip(_E2M1_THRESHOLDS, _E2M1[:-1], _E2M1[1:]):
        mag += (a >= t if tie_up else a > t).to(torch.float32) * (hi - lo)
    return torch.where(v < 0, -mag, mag)


def _blocks(x: torch.Tensor, block: int) -> torch.Tensor:
    return x.float().unflatten(-1, (x.shape[-1] // block, block))


def fp8_qdq(x: torch.Tensor, block: int = 32) -> torch.Tensor:
    """x rounded onto the FP8 grid with one power-of-two scale per `block` values (x's dtype)."""
    b = _blocks(x, block)
    s = pow2_ceil(b.abs().amax(-1, keepdim=True).clamp_min(1e-4) * RECIP_E4M3_MAX)
    return (e4m3(b / s) * s).flatten(-2).to(x.dtype)


def fp4_qdq(x: torch.Tensor, block: int, scale: str = "pow2") -> torch.Tensor:
    """x rounded onto the FP4 grid with one scale per `block` values: `pow2` (E8M0) or `e4m3` scales."""
    b = _blocks(x, block)
    amax = b.abs().amax(-1, keepdim=True)
    if scale == "pow2":
        s = pow2_ceil(amax.clamp_min(E2M1_MAX * 2.0 ** -126) * RECIP_E2M1_MAX)
    elif scale == "e4m3":
        s = e4m3(amax.clamp_min(E2M1_MAX * 2.0 ** -9) / E2M1_MAX)
    else:
        raise ValueError(f"unknown FP4 scale kind {scale!r}")
    return (e2m1((b / s).clamp(-E2M1_MAX, E2M1_MAX)) * s).flatten(-2).to(x.dtype)


# ---------------------------------------------------------------------------- row transforms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = (xf.square().mean(-1, keepdim=True) + eps).rsqrt()
    return (xf * inv * w.float()).to(x.dtype)


def rotate(x: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """RoPE on the last 2 len(freqs) dims of x [T, ..., D]: dims (2i, 2i + 1) of that tail turn by the
    fp32 angle position * freqs[i] (clockwise when `inverse`), evaluated in fp64 and rounded once to
    x's dtype."""
    n = freqs.numel()
    ang = (positions.float()[:, None] * freqs.float()[None]).double()  # fp32 product, then exact
    c, s = torch.cos(ang).float().double(), torch.sin(ang).float().double()  # fp32 cos / sin
    if inverse:
        s = -s
    shape = (positions.shape[0],) + (1,) * (x.dim() - 2) + (n,)
    c, s = c.view(shape), s.view(shape)
    tail = x[..., -2 * n:].double().unflatten(-1, (n, 2))
    re, im = tail[..., 0], tail[..., 1]
    turned = torch.stack((re * c - im * s, re * s + im * c), -1).flatten(-2)
    return torch.cat((x[..., :-2 * n], turned.to(x.dtype)), -1)


def window_kv(kv: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """The cached window row of each token: its kv row [T, 512] rotated by its position, FP8 per 32."""
    return fp8_qdq(rotate(kv, positions, freqs), 32)


def pooled_pair(first: torch.Tensor, second: torch.Tensor, norm_w: torch.Tensor, eps: float) -> torch.Tensor:
    """Ratio-2 group latent from its two tokens' fp32 [kv | score] rows [n, 2 d]: per channel the kv
    values weighted by softmax over the two scores, rounded to bf16, RMS-normalised."""
    d = first.shape[-1] // 2
    a, b = first[..., d:].float(), second[..., d:].float()
    top = torch.maximum(a, b)
    ea, eb = torch.exp(a - top), torch.exp(b - top)
    pooled = (first[..., :d].float() * ea + second[..., :d].float() * eb) / (ea + eb)
    return rms_norm(pooled.to(torch.bfloat16), norm_w, eps)


def compressed_kv(latent: torch.Tensor, group_pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """A closed group's attention row: its latent rotated by the group's first position, FP4 with
    E4M3 scales per 16."""
    return fp4_qdq(rotate(latent, group_pos, freqs), 16, "e4m3")


def index_key(k: torch.Tensor, k_norm: torch.Tensor, group_pos: torch.Tensor, freqs: torch.Tensor,
              eps: float) -> torch.Tensor:
    """A closed group's index key: RMS-normalised wk(latent), rotated, FP4 with power-of-two scales per 32."""
    return fp4_qdq(rotate(rms_norm(k, k_norm, eps), group_pos, freqs), 32, "pow2")


def index_q(q: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """The index query [T, H, 128]: rotated, FP4 with power-of-two scales per 32."""
    return fp4_qdq(rotate(q, positions, freqs), 32, "pow2")


def finish_output(o: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """The per-head attention output [T, h, 512] as wo_a reads it: tail rotated back, FP8 per 32 (the
    32-value blocks never straddle two heads, so the qdq grouping of heads does not matter)."""
    return fp8_qdq(rotate(o, positions, freqs, inverse=True), 32)


# ---------------------------------------------------------------------------- indexer
def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def indexer_scores(qi: torch.Tensor, wi: torch.Tensor, keys: torch.Tensor, n_vis: torch.Tensor,
                   heads_per_group: int) -> torch.Tensor:
    """Scores [n, N] (fp32 holding bf16 values; -inf past each query's n_vis) of query i against its
    own keys[i] [N, D]: qi [n, H, D], wi [n, H] (bf16), heads in rank groups of `heads_per_group`."""
    n, H, _ = qi.shape
    N = keys.shape[1]
    terms = _bf16(torch.relu(_bf16(torch.matmul(qi.float(), keys.float().transpose(1, 2)))) * wi.float()[..., None])
    groups = terms.view(n, H // heads_per_group, heads_per_group, N)
    acc = groups[:, :, 0]
    for j in range(1, heads_per_group):  # head order inside every rank group at once, fp32
        acc = acc + groups[:, :, j]
    per_rank = _bf16(acc)  # [n, R, N]
    total = per_rank[:, 0]
    for r in range(1, per_rank.shape[1]):  # the all-reduce: rank order, bf16 after each addition
        total = _bf16(total + per_rank[:, r])
    visible = torch.arange(N, device=qi.device)[None] < n_vis[:, None]
    return total.masked_fill(~visible, float("-inf"))


def _order_keys(scores: torch.Tensor) -> torch.Tensor:
    """int64 keys whose ascending order is (score descending, column ascending)."""
    # + 0.0 turns -0.0 into +0.0: the two zeros are one score (a tie broken by column)
    bits = (scores.float() + 0.0).contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    # fp32 bit patterns -> unsigned integers that grow with the value (negatives reversed)
    ordered = torch.where(bits >= 0x80000000, 0xFFFFFFFF - bits, bits | 0x80000000)
    col = torch.arange(scores.shape[-1], device=scores.device, dtype=torch.int64)
    return ((0xFFFFFFFF - ordered) << 31) | col  # columns < 2^31


def _best_ascending(keys: torch.Tensor, count: torch.Tensor, k: int) -> torch.Tensor:
    """Per row the columns of the min(k, count) smallest keys, ascending, -1 padded to k."""
    n, N = keys.shape
    out = torch.full((n, k), -1, dtype=torch.int32, device=keys.device)
    w = min(k, N)
    if n == 0 or w == 0:
        return out
    cols = torch.topk(keys, w, dim=-1, largest=False, sorted=True).values & 0x7FFFFFFF
    taken = torch.arange(w, device=keys.device)[None] < count[:, None]
    cols = torch.sort(torch.where(taken, cols, N), -1).values
    out[:, :w] = torch.where(cols == N, -1, cols).to(torch.int32)
    return out


def select_topk(scores: torch.Tensor, n_vis: torch.Tensor, k: int) -> torch.Tensor:
    """The chosen groups per query: the min(k, n_vis) best visible columns, ascending, -1 padded."""
    keys = _order_keys(scores)
    N = scores.shape[-1]
    visible = torch.arange(N, device=scores.device)[None] < n_vis[:, None]
    keys = torch.where(visible, keys, torch.iinfo(torch.int64).max)
    return _best_ascending(keys, n_vis.clamp(0, N), k)


def pick_blocks(scores: torch.Tensor, n_vis: torch.Tensor, topk_blocks: int, block: int) -> torch.Tensor:
    """Blocks of `block` groups ranked by their best score (the newest visible group's block first),
    the best `topk_blocks` among blocks holding a visible group, ascending, -1 padded."""
    n, N = scores.shape
    nb = -(-N // block)
    padded = torch.full((n, nb * block), float("-inf"), device=scores.device)
    padded[:, :N] = scores
    best = padded.view(n, nb, block).amax(-1)
    newest = torch.div(n_vis - 1, block, rounding_mode="floor")
    best = torch.where(torch.arange(nb, device=scores.device)[None] == newest[:, None], float("inf"), best)
    reachable = torch.div(n_vis + block - 1, block, rounding_mode="floor")
    keys = torch.where(torch.arange(nb, device=scores.device)[None] < reachable[:, None], _order_keys(best),
                       torch.iinfo(torch.int64).max)
    return _best_ascending(keys, reachable, topk_blocks)


def restrict_to_blocks(scores: torch.Tensor, blocks: torch.Tensor, block: int) -> torch.Tensor:
    """Scores with every visible group outside the listed blocks (-1 = none) set to -FLT_MAX."""
    col_block = torch.arange(scores.shape[-1], device=scores.device) // block
    member = (blocks.long()[:, :, None] == col_block[None, None, :]).any(1)
    return torch.where(member | torch.isneginf(scores), scores, NEG_FLT_MAX)


# ---------------------------------------------------------------------------- attention
def attend_with_sink(q: torch.Tensor, rows: torch.Tensor, valid: torch.Tensor, sink: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """q [n, h, d] over rows [n, R, d] (K = V; valid [n, R]) with a per-head sink [h] -> [n, h, d] bf16."""
    logits = torch.matmul(q.float(), rows.float().transpose(1, 2)) * scale  # [n, h, R]
    logits = logits.masked_fill(~valid[:, None, :], float("-inf"))
    has = valid.any(-1)
    top = torch.where(has[:, None], logits.amax(-1), 0.0)  # [n, h]; any finite value without rows
    e = torch.exp(logits - top[..., None])
    den = e.sum(-1) + torch.exp(sink.float()[None] - top)
    out = torch.matmul(_bf16(e), rows.float()) / den[..., None]
    return torch.where(has[:, None, None], out, 0.0).to(torch.bfloat16)
