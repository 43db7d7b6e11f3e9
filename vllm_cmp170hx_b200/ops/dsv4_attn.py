"""DeepSeek-V4.1 attention core: window + compressed KV, indexer top-k, sparse attention with sinks.

`DSv4AttnCore` holds one layer's caches and runs a step over any mix of prefill chunks and decode
tokens.  B200 layout: every row a query can attend -- the compressed group rows (paged on the
engine's token blocks), the sliding-window rings and this step's own window rows -- lives in ONE
bf16 pool, so the attention is a single gather over pool row ids and runs on the tcgen05
block-sparse attention kernel (csrc/mla_attn.cu, 512-wide rows, per-head sink in the softmax
denominator).

Rounding points and selection rules are the reference's (oracle/dsv4_attn.py states them; the
reference's layer is vllm_sm80/models/deepseek_v41/ops/sm80_attn_core.py:783 prepare_layer and
:848 attend_layer).  On the GPU the index scores run on csrc/dsv4_index.cu (the same rounding chain over
the paged group keys) and the selection on the canonical top-k kernel; the two-level candidate-block
selection, the RoPE turns and the FP8 / FP4 qdq steps on csrc/dsv4_rot.cu (one pass per row); the
ratio-2 pooling and the ring bookkeeping run as torch ops on the step's tensors; on CPU tensors everything
runs on the oracle.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _ext
from ..oracle import dsv4_attn as ref


_ROT_MODES = {"none": 0, "fp8": 1, "fp4_e4m3": 2, "fp4_pow2": 3}


def rot_qdq(x: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor, mode: str, inverse: bool = False,
            norm_w: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """The row transforms of the layer on x [T, D] or [T, heads, D] (bf16): optional RMSNorm, the RoPE turn of
    the tail at each token's position, then the qdq `mode` ("none", "fp8" per 32, "fp4_e4m3" per 16,
    "fp4_pow2" per 32).  CUDA: csrc/dsv4_rot.cu in one pass; CPU: the oracle's functions."""
    if not x.is_cuda:
        y = ref.rms_norm(x, norm_w, eps) if norm_w is not None else x
        y = ref.rotate(y, positions, freqs, inverse=inverse)
        if mode == "fp8":
            return ref.fp8_qdq(y, 32)
        if mode == "fp4_e4m3":
            return ref.fp4_qdq(y, 16, "e4m3")
        if mode == "fp4_pow2":
            return ref.fp4_qdq(y, 32, "pow2")
        return y
    heads = x.shape[1] if x.dim() == 3 else 1
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty(x2.shape, dtype=torch.bfloat16, device=x.device)
    _ext.ops().dsv4_rot_qdq(x2.to(torch.bfloat16), out, positions.to(torch.int64).contiguous(), heads,
                            freqs.float().contiguous(), inverse, norm_w, eps, _ROT_MODES[mode])
    return out.view(x.shape)


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
        return ref.attend_with_sink(q, pool[idx.clamp_min(0).long()], idx >= 0, sink, scale)
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
    """One layer's caches and step.  Pool rows: [groups | rings | step scratch]:

    * groups (and index keys): one row per closed group, paged like the engine's token blocks --
      group g of sequence s at block_table[s, g // 64] * 64 + g % 64 (g <= position, so the block is
      always allocated);
    * rings: `window` (+ the speculative width) rows per sequence slot, position p at row p % ring;
    * scratch: this step's window rows in token order, which the step's queries read for positions
      inside the step (the ring keeps earlier positions); after the attention the last `ring`
      positions of each sequence move into its ring.
    """

    def __init__(self, spec: DSv4AttnSpec, num_slots: int, group_rows: int, max_step_tokens: int,
                 freqs: torch.Tensor, sink: torch.Tensor, comp_norm: torch.Tensor | None = None,
                 wk: torch.Tensor | None = None, k_norm: torch.Tensor | None = None, device="cpu",
                 carry_rows: int = 2, ring_extra: int = 0):
        self.spec, self.device = spec, torch.device(device)
        d = spec.head_dim
        # ring rows per slot: the window plus the positions a speculative verify step may write past
        # the accepted ones (without them a rejected draft would evict a row the window still needs)
        self.ring = spec.window + ring_extra
        self.G0, self.W0 = 0, group_rows
        self.S0 = group_rows + num_slots * self.ring
        self.max_step = max_step_tokens
        # one dummy row past the scratch (pool) and past the groups (index keys): masked writes of
        # tokens that write nothing land there, so no step needs a data-dependent shape
        self.dummy = self.S0 + max_step_tokens
        self.pool = torch.zeros(self.dummy + 1, d, dtype=torch.bfloat16, device=self.device)
        self.kdummy = max(group_rows, 1)
        self.idxk = torch.zeros(self.kdummy + 1, spec.index_dim, dtype=torch.bfloat16, device=self.device)
        # ratio 2: the raw fp32 [kv | score] rows of each slot's last `carry_rows` positions (a step
        # that starts on a group's second token pools it with the row before; speculative verify steps
        # need as many rows as their width + 1, since rejected positions are written too)
        self.carry = max(2, carry_rows)
        self.prev = torch.zeros(num_slots + 1, self.carry, 2 * d, dtype=torch.float32, device=self.device)
        self.freqs = freqs.float().to(self.device)
        self.sink = sink.float().to(self.device)
        self.comp_norm, self.wk, self.k_norm = comp_norm, wk, k_norm

    def _group_rows(self, block_table: torch.Tensor, seq: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        return block_table[seq.long(), (g // 64).long()].long() * 64 + g.long() % 64

    # ------------------------------------------------------------------ compressed groups
    def _write_groups(self, seq, slot, pos, kv, kv_score, block_table, valid=None):
        sp = self.spec
        if sp.ratio == 1:
            # the compressor's own bf16 row when given (kv_score), else the attention's kv row
            closes = torch.ones_like(pos, dtype=torch.bool)
            latent = ref.rms_norm(kv_score if kv_score is not None else kv, self.comp_norm, sp.eps)
        else:
            closes = (pos + 1) % 2 == 0
            # the group's first row: the previous token of this step, or the sequence's open row
            same = torch.zeros_like(closes)
            same[1:] = (seq[1:] == seq[:-1]) & (pos[1:] == pos[:-1] + 1)
            tslot = slot[seq.long()].long()
            carried = self.prev[tslot, (pos - 1) % self.carry]
            prev = torch.where(same[:, None], torch.roll(kv_score, 1, 0), carried)
            latent = ref.pooled_pair(prev, kv_score, self.comp_norm, sp.eps)
            # the last `carry` positions of each sequence into its carry ring (distinct rows; the
            # others into the dummy slot)
            keep = pos > self._last_pos(seq, pos, slot.shape[0]) - self.carry
            if valid is not None:
                keep = keep & valid
            dslot = self.prev.shape[0] - 1
            self.prev[torch.where(keep, tslot, dslot), torch.where(keep, pos % self.carry, 0)] = kv_score.float()
        if valid is not None:
            closes = closes & valid
        g = (torch.div(pos + 1, sp.ratio, rounding_mode="floor") - 1).clamp_min(0)
        gpos = pos + 1 - sp.ratio
        rows = self._group_rows(block_table, seq, g)
        self.pool[torch.where(closes, self.G0 + rows, self.dummy)] = rot_qdq(latent, gpos, self.freqs, "fp4_e4m3")
        if latent.is_cuda:
            from . import gemm

            k = gemm(latent.to(torch.bfloat16), self.wk.to(torch.bfloat16))  # fp32 accumulate, bf16 out
            self.idxk[torch.where(closes, rows, self.kdummy)] = rot_qdq(k, gpos, self.freqs, "fp4_pow2", False,
                                                                         self.k_norm.to(torch.bfloat16), sp.eps)
            return
        k = latent.float() @ self.wk.float().t()
        self.idxk[torch.where(closes, rows, self.kdummy)] = ref.index_key(k.to(torch.bfloat16), self.k_norm, gpos,
                                                                          self.freqs, sp.eps)

    @staticmethod
    def _last_pos(seq: torch.Tensor, pos: torch.Tensor, S: int) -> torch.Tensor:
        """Per token, the last position its sequence reaches in this step."""
        last = torch.full((S,), -1, dtype=torch.long, device=pos.device)
        last.scatter_reduce_(0, seq.long(), pos.long(), reduce="amax", include_self=True)
        return last[seq.long()]

    # ------------------------------------------------------------------ one step
    def step(self, seq: torch.Tensor, pos: torch.Tensor, slot: torch.Tensor, block_table: torch.Tensor,
             q: torch.Tensor, kv: torch.Tensor, kv_score: torch.Tensor | None = None,
             index_q: torch.Tensor | None = None, index_w: torch.Tensor | None = None,
             candidates_in: torch.Tensor | None = None, candidates_out: list | None = None,
             max_groups: int | None = None, valid: torch.Tensor | None = None) -> torch.Tensor:
        """Tokens of this step, each sequence's tokens consecutive and in position order: seq [T]
        (row of block_table / slot), pos [T]; slot [S] ring slot of each sequence; q [T, h, 512]
        (pre-RoPE), kv [T, 512] (kv_norm(wkv(x)), pre-RoPE), kv_score [T, 1024] fp32 (ratio 2; at ratio 1 an optional bf16 [T, 512]),
        index_q [T, H_i, 128] (pre-RoPE), index_w [T, H_i] (weights_proj(x)); max_groups: a host
        bound on any token's visible groups (the indexer's score width; None reads it from the
        device).  With max_groups given the step reads no device value on the host (graph
        capturable).  valid [T] bool: tokens that write cache rows (padding tokens of a CUDA-graph batch
        carry another sequence's index and must leave its groups, rings and carry rows alone); None: all.
        Returns the wo_a input [T, h, 512]."""
        sp = self.spec
        T = pos.shape[0]
        if T > self.max_step:
            raise ValueError(f"{T} tokens in a step, the scratch holds {self.max_step}")
        dev = pos.device
        pos = pos.long()
        seq_l = seq.long()
        wrows = rot_qdq(kv, pos, self.freqs, "fp8")
        self.pool[self.S0:self.S0 + T] = wrows
        if sp.ratio:
            self._write_groups(seq, slot, pos, kv, kv_score, block_table, valid)
        # first token and position of each token's sequence within this step
        tix = torch.arange(T, device=dev)
        new = torch.ones(T, dtype=torch.bool, device=dev)
        new[1:] = seq_l[1:] != seq_l[:-1]
        first = torch.cummax(torch.where(new, tix, 0), 0).values
        p0 = pos[first]
        # window rows of positions [p - window + 1, p]: this step's from the scratch, earlier ones
        # from the sequence's ring
        back = torch.arange(sp.window, device=dev)
        wpos = pos[:, None] - back[None]
        in_step = wpos >= p0[:, None]
        ring = self.W0 + slot[seq_l].long()[:, None] * self.ring + wpos % self.ring
        scratch = self.S0 + first[:, None] + (wpos - p0[:, None])
        widx = torch.where(wpos < 0, -1, torch.where(in_step, scratch, ring))
        idx = [widx]
        if sp.ratio:
            n_vis = torch.div(pos + 1, sp.ratio, rounding_mode="floor")
            qi = rot_qdq(index_q, pos, self.freqs, "fp4_pow2")
            wi = (index_w.float() * (sp.index_dim ** -0.5 * sp.index_heads ** -0.5)).to(torch.bfloat16)
            N = max(1, max_groups if max_groups is not None else int(n_vis.max()))
            if q.is_cuda and not sp.candidate_blocks and candidates_in is None:
                # the scores kernel (csrc/dsv4_index.cu: the rounding chain of ref.indexer_scores over the
                # paged group keys) and the canonical top-k kernel, straight to group rows through the
                # block table -- no gathered key tensor, no sorts
                ops = _ext.ops()
                scores = torch.empty(T, N, dtype=torch.float32, device=dev)
                nv = n_vis.to(torch.int32)
                sq = seq_l.to(torch.int32)
                bt = block_table.to(torch.int32).contiguous()  # the engine's is int32 already
                ops.dsv4_index_scores(qi.to(torch.bfloat16).contiguous(), wi.contiguous(), self.idxk, bt,
                                      sq, nv, sp.index_heads_per_rank, scores)
                top = torch.empty(T, sp.index_topk, dtype=torch.int32, device=dev)
                cnt = torch.empty(T, dtype=torch.int32, device=dev)
                ops.mla_topk(scores, nv, sp.index_topk, sq, bt, 64, top, cnt)
                idx.append(torch.where(top >= 0, self.G0 + top.long(), -1))
                N = 0  # nothing left for the host selection below
            # every query scores the groups of its own sequence, in row chunks of bounded size
            per_row = max(N, 1) * (sp.index_heads * 4 + sp.index_dim * 2 + 16)
            rc = max(1, (256 << 20) // per_row)
            gi = torch.arange(N, device=dev)
            sels, cbs = [], []
            for r0 in range(0, T if N else 0, rc):
                r = slice(r0, min(T, r0 + rc))
                gr = block_table[seq_l[r]][:, gi // 64].long() * 64 + gi % 64  # [rows, N] group rows
                scores = ref.indexer_scores(qi[r], wi[r], self.idxk[gr], n_vis[r], sp.index_heads_per_rank)
                if sp.candidate_blocks and candidates_in is None:
                    cbs.append(ref.pick_blocks(scores, n_vis[r], sp.candidate_blocks, sp.candidate_block))
                elif candidates_in is not None:
                    scores = ref.restrict_to_blocks(scores, candidates_in[r], sp.candidate_block)
                top = ref.select_topk(scores, n_vis[r], sp.index_topk).long()
                sels.append(torch.where(top >= 0, self.G0 + gr.gather(1, top.clamp_min(0)), -1))
            if candidates_out is not None and cbs:
                candidates_out.append(torch.cat(cbs))
            if sels:
                idx.append(torch.cat(sels))
        qr = rot_qdq(q, pos, self.freqs, "none")
        o = attend(qr, self.pool, torch.cat(idx, 1), self.sink, sp.head_dim ** -0.5)
        # the last `ring` positions of each sequence into its ring (distinct ring rows; the others
        # into the dummy row)
        keep = pos > self._last_pos(seq_l, pos, slot.shape[0]) - self.ring
        if valid is not None:
            keep = keep & valid
        ring_rows = self.W0 + slot[seq_l].long() * self.ring + pos % self.ring
        self.pool[torch.where(keep, ring_rows, self.dummy)] = wrows
        return rot_qdq(o, pos, self.freqs, "fp8", inverse=True)
