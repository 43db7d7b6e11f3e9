"""DeepSeek-V4.1 attention core: window + compressed KV, indexer top-k, sparse attention with sinks.

`DSv4AttnCore` holds one layer's caches for up to `max_seqs` sequences and runs a step over any
mix of prefill chunks and decode tokens.  B200 layout: every row a query can attend -- the
sliding-window rows and the compressed group rows -- lives in ONE bf16 pool [max_seqs * R, 512]
(per sequence a window ring of `window + max_chunk` rows, then one row per group), so the attention
is a single gather over pool row ids and runs on the tcgen05 block-sparse attention kernel
(csrc/mla_attn.cu, 512-wide rows, per-head sink in the softmax denominator).  The ring is wider than
the window by the largest chunk, so no row a query of the chunk needs is overwritten by the chunk.

Rounding points and selection rules are the reference's (oracle/dsv4_attn.py states them; the
reference's layer is vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py:783 prepare_layer and
:848 attend_layer).  Index scores, top-k and the qdq steps run as torch ops on the step's tensors;
on CPU tensors everything runs on the oracle.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _ext
from ..oracle import dsv4_attn as ref


@dataclass
class DSv4AttnSpec:
    heads: int  # query heads on this rank
    head_dim: int = 512
    rope_dim: int = 64
    window: int = 128
    ratio: int = 1  # compression ratio (1 or 2); 0: window only
    index_heads: int = 32
    index_dim: int = 128
    index_topk: int = 512
    index_heads_per_rank: int = 32  # the score rounding groups (index heads / tensor-parallel size)
    out_groups: int = 1  # output qdq groups on this rank
    eps: float = 1e-6
    candidate_blocks: int = 0  # >0: two-level selection over blocks of `candidate_block` groups
    candidate_block: int = 64


def attend(q: torch.Tensor, pool: torch.Tensor, idx: torch.Tensor, sink: torch.Tensor, scale: float,
           splits: int | None = None) -> torch.Tensor:
    """q [T, h, 512] bf16 over pool rows idx [T, R] (int, -1 = none; K = V = the row) with a per-head
    sink [h] fp32 -> [T, h, 512] bf16."""
    if not q.is_cuda:
        return ref.sparse_attention(q, pool[idx.clamp_min(0).long()], idx >= 0, sink, scale)
    from .mla import pick_splits

    # valid rows first (stable), then the per-token count: the kernel reads the first `count`
    order = torch.sort((idx < 0).to(torch.int8), dim=1, stable=True).indices
    packed = idx.gather(1, order).to(torch.int32).contiguous()
    counts = (idx >= 0).sum(1, dtype=torch.int32)
    T, h, _ = q.shape
    out = torch.empty(T, h, 512, dtype=torch.bfloat16, device=q.device)
    s = splits if splits is not None else pick_splits(T, h, packed.shape[1])
    _ext.ops().mla_sparse_attention(q.contiguous(), pool, packed, counts, float(scale), s, out, None,
                                    _ext.status_word(q.device), sink.float().contiguous())
    return out


class DSv4AttnCore:
    def __init__(self, spec: DSv4AttnSpec, max_seqs: int, max_len: int, max_chunk: int, freqs: torch.Tensor,
                 sink: torch.Tensor, comp_norm: torch.Tensor | None = None, wk: torch.Tensor | None = None,
                 k_norm: torch.Tensor | None = None, device="cpu"):
        self.spec, self.device = spec, torch.device(device)
        self.max_chunk = max_chunk
        self.ring = spec.window + max_chunk
        self.groups = max_len // spec.ratio if spec.ratio else 0
        self.R = self.ring + self.groups
        d = spec.head_dim
        self.pool = torch.zeros(max_seqs * self.R, d, dtype=torch.bfloat16, device=self.device)
        self.idxk = torch.zeros(max_seqs, max(self.groups, 1), spec.index_dim, dtype=torch.bfloat16,
                                device=self.device)
        self.prev = torch.zeros(max_seqs, 2 * d, dtype=torch.float32, device=self.device)  # open ratio-2 group
        self.freqs = freqs.float().to(self.device)
        self.sink = sink.float().to(self.device)
        self.comp_norm, self.wk, self.k_norm = comp_norm, wk, k_norm

    # ------------------------------------------------------------------ cache writes
    def _write(self, seq: torch.Tensor, pos: torch.Tensor, kv: torch.Tensor, kv_score: torch.Tensor | None):
        sp = self.spec
        base = seq.long() * self.R
        self.pool[base + pos.long() % self.ring] = ref.window_rows(kv, pos, self.freqs)
        if not sp.ratio:
            return
        if sp.ratio == 1:
            closes = torch.ones_like(pos, dtype=torch.bool)
            latent = ref.rms_norm(kv, self.comp_norm, sp.eps)
        else:
            closes = (pos + 1) % 2 == 0
            # the group's first row: the previous token of this chunk, or the sequence's open row
            same = torch.zeros_like(closes)
            same[1:] = (seq[1:] == seq[:-1]) & (pos[1:] == pos[:-1] + 1)
            prev = torch.where(same[:, None], torch.roll(kv_score, 1, 0), self.prev[seq.long()])
            latent = ref.pool_pair(prev, kv_score, self.comp_norm, sp.eps)
            # a sequence whose chunk ends on a group's first token keeps that row for the next step
            last = torch.ones_like(closes)
            last[:-1] = seq[1:] != seq[:-1]
            keep = last & ~closes
            self.prev[seq[keep].long()] = kv_score[keep].float()
        g = torch.div(pos + 1, sp.ratio, rounding_mode="floor") - 1
        gpos = pos + 1 - sp.ratio
        c = closes.nonzero().flatten()
        if c.numel() == 0:
            return
        sc, gc = seq[c].long(), g[c].long()
        self.pool[sc * self.R + self.ring + gc] = ref.compressed_rows(latent[c], gpos[c], self.freqs)
        k = latent[c].float() @ self.wk.float().t()
        self.idxk[sc, gc] = ref.index_key_rows(k.to(torch.bfloat16), self.k_norm, self.freqs, gpos[c], sp.eps)

    # ------------------------------------------------------------------ one step
    def step(self, seq: torch.Tensor, pos: torch.Tensor, q: torch.Tensor, kv: torch.Tensor,
             kv_score: torch.Tensor | None = None, index_q: torch.Tensor | None = None,
             index_w: torch.Tensor | None = None, candidates_in: torch.Tensor | None = None,
             candidates_out: list | None = None) -> torch.Tensor:
        """Tokens of this step (each sequence's tokens consecutive and in position order, at most
        `max_chunk` per sequence): seq [T], pos [T], q [T, h, 512] (pre-RoPE), kv [T, 512]
        (kv_norm(wkv(x)), pre-RoPE), kv_score [T, 1024] fp32 (ratio 2), index_q [T, H_i, 128]
        (pre-RoPE), index_w [T, H_i] (weights_proj(x)).  Returns the wo_a input [T, h, 512]."""
        sp = self.spec
        T = pos.shape[0]
        self._write(seq, pos, kv, kv_score)
        # window rows of positions [p - window + 1, p]
        back = torch.arange(sp.window, device=pos.device)
        wpos = pos[:, None] - back[None]
        widx = torch.where(wpos >= 0, seq[:, None].long() * self.R + wpos % self.ring, -1)
        idx = [widx]
        if sp.ratio:
            n_vis = torch.div(pos + 1, sp.ratio, rounding_mode="floor")
            qi = ref.index_query(index_q, pos, self.freqs)
            wi = (index_w.float() * (sp.index_dim ** -0.5 * sp.index_heads ** -0.5)).to(torch.bfloat16)
            sel = torch.full((T, sp.index_topk), -1, dtype=torch.long, device=pos.device)
            cands = []
            for s in torch.unique(seq).tolist():
                rows = (seq == s).nonzero().flatten()
                N = max(int(n_vis[rows].max()), 1)
                scores = ref.index_scores(qi[rows], wi[rows], self.idxk[s, :N], n_vis[rows], sp.index_heads_per_rank)
                if sp.candidate_blocks and candidates_in is None:
                    cands.append((rows, ref.candidate_blocks(scores, n_vis[rows], sp.candidate_blocks,
                                                             sp.candidate_block)))
                elif candidates_in is not None:
                    scores = ref.mask_to_candidates(scores, candidates_in[rows], sp.candidate_block)
                top = ref.topk_canonical(scores, n_vis[rows], sp.index_topk).long()
                sel[rows] = torch.where(top >= 0, s * self.R + self.ring + top, -1)
            if candidates_out is not None and cands:
                out = torch.full((T, sp.candidate_blocks), -1, dtype=torch.int32, device=pos.device)
                for rows, c in cands:
                    out[rows] = c
                candidates_out.append(out)
            idx.append(sel)
        qr = ref.rope(q, pos, self.freqs)
        o = attend(qr, self.pool, torch.cat(idx, 1), self.sink, sp.head_dim ** -0.5)
        return ref.output_qdq(o, pos, self.freqs, sp.out_groups)
