"""Hybrid KDA / sparse-MLA MoE causal LM (the GLM-5.3-Flash family of the
reference, vllm_sm80/models/glm5next/sm80_model.py:112-434, in the shapes of
BASELINE config 3), and the DeepSeek-style all-MLA variant (config 4) through
the same classes.

Per layer: RMSNorm -> attention (KDA or sparse MLA) -> row-parallel
projection + TP all-reduce -> fused residual-add RMSNorm -> MoE (router,
routed experts, shared expert) or dense MLP -> TP all-reduce.

Tensor parallel: attention heads and expert intermediates are split across
the TP group (whole H128 blocks for EXL3 experts, as the reference's
`aligned_shard`, vllm_sm80/kernels/exl3/utils.py:146); the indexer, router
and embedding are replicated; the LM head is vocab-parallel and sampling
combines per-rank winners without gathering logits.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
from torch import nn

from .. import ops
from ..config import ModelConfig
from ..formats import exl3 as fx
from ..ops import kda as kda_ops
from ..ops import mhc as mhc_ops
from ..ops import mla as mla_ops
from ..ops import moe as moe_ops
from ..oracle import mla as mla_ref
from ..parallel import comm
from ..parallel import state as pstate
from ..parallel.sp import scope as sp_scope
from .layers import Linear, RMSNorm, WeightInit, default_std


@dataclass
class StepContext:
    """Device tensors describing one forward batch (built by the runner)."""

    positions: torch.Tensor  # [T] int32
    num_tokens: int
    # sparse-MLA (paged latent cache, block 64)
    slot_mapping: torch.Tensor | None = None  # [T] int64 cache rows of the new tokens
    token_seq: torch.Tensor | None = None  # [T] int32 sequence index of each token
    ctx_lens: torch.Tensor | None = None  # [T] int32 visible positions (pos + 1)
    block_table: torch.Tensor | None = None  # [S, max_blocks] int32
    max_ctx: int = 0  # host bound of ctx_lens (indexer score width)
    # KDA (per-sequence recurrent state slots)
    cu_seqlens: torch.Tensor | None = None  # [S + 1] int32
    kda_slots: torch.Tensor | None = None  # [S] int32
    has_init: torch.Tensor | None = None  # [S] int32
    # caches, by layer index
    mla_caches: dict = field(default_factory=dict)  # i -> (latent [rows, 576], idx_k [rows, 128] u8, idx_s [rows])
    kda_states: dict = field(default_factory=dict)  # i -> (rec [slots, H, 128, 128] f32, conv [slots, 3HD, 3])
    scores_buf: torch.Tensor | None = None
    # speculative verify of models with KDA layers: int32 [S] (1 = the sequence's state is only
    # recorded, see HybridForCausalLM.kda_recover) and the per-layer records of the step
    kda_verify: torch.Tensor | None = None
    kda_records: dict = field(default_factory=dict)
    # DeepSeek-V4.1 attention layers: i -> DSv4AttnCore (caches; rings indexed by kda_slots)
    dsa_cores: dict = field(default_factory=dict)
    # gated grouped-query attention layers: i -> paged [k | v] rows [positions * kv heads, 512] bf16
    gqa_caches: dict = field(default_factory=dict)
    # n-gram embedding ids of the step's tokens, int64 [T, heads] (models with a PLE table)
    ple_ids: torch.Tensor | None = None
    # Engram memory ids of the step's tokens, int64 [T, heads], and the rows the stage looked up for them
    engram_ids: torch.Tensor | None = None
    engram_rows: torch.Tensor | None = None
    engram_ready: object = None  # CUDA event of the side-stream lookup (None: rows ready in stream order)


def _fp8_proj(w: torch.Tensor):
    from .marlin_experts import Fp8Proj

    return Fp8Proj(w)


# ============================================================================ attention
class KDAAttention(nn.Module):
    """Kimi-delta attention layer (GLM `linear_attention`): fused input GEMM
    [q | k | v | f_a | g_a | beta], low-rank gate up-projections f_b / g_b, the
    fused conv + gates + recurrence + gated-norm kernel, row-parallel o_proj."""

    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        k = cfg.kda
        H, D = k.num_heads, k.head_dim
        assert H % tp == 0 and D == 128
        self.H = H // tp
        self.D = D
        self.lower_bound = k.lower_bound
        hid = cfg.hidden_size
        HD = self.H * D
        sd = default_std(hid)
        # fused input projection: q, k, v (this rank's heads) | f_a | g_a (replicated rank-D) | beta
        wq = wi.normal((H * D, hid), sd, (0, tp_rank, tp))
        wk = wi.normal((H * D, hid), sd, (0, tp_rank, tp))
        wv = wi.normal((H * D, hid), sd, (0, tp_rank, tp))
        wfa = wi.normal((D, hid), sd)
        wga = wi.normal((D, hid), sd)
        wb = wi.normal((H, hid), sd, (0, tp_rank, tp))
        rows = 3 * HD + 2 * D + self.H
        pad = (-rows) % 8  # keep the fused output's row stride 16-byte aligned (TMA)
        wpad = torch.zeros(pad, hid, dtype=wq.dtype, device=wq.device)
        self.in_proj = Linear(torch.cat([wq, wk, wv, wfa, wga, wb, wpad], dim=0).contiguous())
        self.f_b = Linear(wi.normal((H * D, D), default_std(D), (0, tp_rank, tp)))
        self.g_b = Linear(wi.normal((H * D, D), default_std(D), (0, tp_rank, tp)))
        self.conv_w = nn.Parameter(wi.normal((3 * H * D, 4), 0.5, None).view(3, H, D, 4)[:, tp_rank * self.H:
                                   (tp_rank + 1) * self.H].reshape(3 * HD, 4).contiguous(), requires_grad=False)
        self.a_log = nn.Parameter(wi.uniform((H,), -1.0, 1.0)[tp_rank * self.H:(tp_rank + 1) * self.H].contiguous(),
                                  requires_grad=False)
        self.g_bias = nn.Parameter(wi.uniform((H * D,), -0.1, 0.1)[tp_rank * HD:(tp_rank + 1) * HD].contiguous(),
                                   requires_grad=False)
        self.norm_w = nn.Parameter(wi.ones_plus(D, 0.05), requires_grad=False)
        self.o_proj = Linear(wi.normal((hid, H * D), default_std(H * D), (1, tp_rank, tp)))

    def forward(self, x: torch.Tensor, ctx: StepContext, layer_idx: int) -> torch.Tensor:
        rec, conv = ctx.kda_states[layer_idx]
        proj = self.in_proj(x)
        HD = self.H * self.D
        qkv = proj[:, : 3 * HD]
        fa = proj[:, 3 * HD: 3 * HD + self.D]
        ga = proj[:, 3 * HD + self.D: 3 * HD + 2 * self.D]
        beta = proj[:, 3 * HD + 2 * self.D: 3 * HD + 2 * self.D + self.H]
        g_raw = self.f_b(fa)
        g2 = self.g_b(ga)
        records = None
        if ctx.kda_verify is not None:
            records = ctx.kda_records.setdefault(layer_idx, kda_ops.KdaRecords())
        o = kda_ops.kda_forward(qkv, g_raw, beta, g2, ctx.cu_seqlens, ctx.kda_slots, ctx.has_init, conv, self.conv_w,
                                None, self.a_log, self.g_bias, self.lower_bound, self.norm_w, rec,
                                verify=ctx.kda_verify, records=records)
        return self.o_proj.forward_reduced(o)


class MLAAttention(nn.Module):
    """DeepSeek-V3.2-style sparse MLA with the lightning indexer
    (vllm_sm80/models/glm5next/sm80_mla.py, sm80_indexer.py): absorbed
    q_nope, paged latent cache (block 64), fp8 indexer top-k, latent
    attention over the selected rows, per-head V up-projection, o_proj."""

    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        m = cfg.mla
        self.m = m
        hid = cfg.hidden_size
        assert m.num_heads % tp == 0
        self.H = m.num_heads // tp
        self.eps = cfg.rms_eps
        from .. import envs

        # With expert parallelism every rank holds all heads (bf16 projections): steps in the
        # sequence-parallel layout attend data-parallel (each rank its own tokens, all heads, no
        # collective), steps in the replicated layout use this rank's head slice [h0, h0 + H).
        self.full_heads = (tp > 1 and pstate.get().expert_parallel and m.attn_weight_format != "fp8_block"
                           and envs.get("VLLM_B200_MLA_DP"))
        self.H_all = m.num_heads if self.full_heads else self.H
        self.h0 = tp_rank * self.H if self.full_heads else 0
        if self.full_heads:
            tp, tp_rank = 1, 0
        sd = default_std(hid)
        ql, kvl = m.q_lora_rank, m.kv_lora_rank
        self.ql, self.kvl = ql, kvl
        dn, dr, dv = m.qk_nope_head_dim, m.qk_rope_head_dim, m.v_head_dim
        self.dn, self.dr, self.dv = dn, dr, dv
        assert kvl == 512 and dr == 64 and m.index_head_dim == 128
        # fused first projection: q_a | kv_a (512 + 64) | indexer k (128) | indexer head weights
        self.in_splits = [ql, kvl + dr, m.index_head_dim, m.index_n_heads]
        fp8 = m.attn_weight_format == "fp8_block"
        Proj = _fp8_proj if fp8 else Linear
        if fp8 and tp > 1:
            # a rank's shard of a block-scaled weight must hold whole 128x128 scale blocks
            assert self.H * (dn + dr) % 128 == 0 and self.H * dv % 128 == 0, "fp8 shard not 128-aligned"
        self.in_proj = Proj(torch.cat([wi.normal((ql, hid), sd), wi.normal((kvl + dr, hid), sd),
                                       wi.normal((m.index_head_dim, hid), sd),
                                       wi.normal((m.index_n_heads, hid), sd)], dim=0).contiguous())
        self.q_a_norm = RMSNorm(wi.ones_plus(ql, 0.05), cfg.rms_eps)
        self.kv_a_norm_w = nn.Parameter(wi.ones_plus(kvl, 0.05), requires_grad=False)
        self.q_b = Proj(wi.normal((m.num_heads * (dn + dr), ql), default_std(ql), (0, tp_rank, tp)))
        # kv_b: [H*(dn + dv), kvl] -> per-head W_UK (stored transposed, [H, kvl, dn]: the absorb GEMM's
        # K-major operand) and W_UV ([H, dv, kvl]: the up-projection's)
        kvb = wi.normal((m.num_heads, dn + dv, kvl), default_std(kvl), (0, tp_rank, tp))
        self.w_uk_t = nn.Parameter(kvb[:, :dn, :].transpose(1, 2).contiguous(), requires_grad=False)
        self.w_uv_t = nn.Parameter(kvb[:, dn:, :].contiguous(), requires_grad=False)  # [H, dv, kvl]
        self.o_proj = Proj(wi.normal((hid, m.num_heads * dv), default_std(m.num_heads * dv), (1, tp_rank, tp)))
        # indexer
        self.idx_q = Linear(wi.normal((m.index_n_heads * m.index_head_dim, ql), default_std(ql)))
        self.idx_k_ln_w = nn.Parameter(wi.ones_plus(m.index_head_dim, 0.05), requires_grad=False)
        self.idx_k_ln_b = nn.Parameter(torch.zeros(m.index_head_dim, dtype=torch.bfloat16, device=wi.device),
                                       requires_grad=False)
        self.sm_scale = 1.0 / math.sqrt(dn + dr)
        self.idx_wscale = m.index_n_heads ** -0.5 * m.index_head_dim ** -0.5
        self.register_buffer("cos_sin", mla_ref.rope_cos_sin(min(cfg.max_position, 1 << 17), dr, m.rope_theta,
                                                             wi.device), persistent=False)

    def forward(self, x: torch.Tensor, ctx: StepContext, layer_idx: int) -> torch.Tensor:
        latent, idx_k, idx_s = ctx.mla_caches[layer_idx]
        T = x.shape[0]
        m = self.m
        proj = self.in_proj(x)
        ql, kvl, dr = self.ql, self.kvl, self.dr
        q_lat = self.q_a_norm(proj[:, :ql])  # the norm reads the strided rows
        kv = proj[:, ql: ql + kvl + dr]
        k_idx = proj[:, ql + kvl + dr: ql + kvl + dr + m.index_head_dim]
        w_idx = proj[:, ql + kvl + dr + m.index_head_dim:]
        pos = ctx.positions
        # caches for the new tokens
        mla_ops.latent_cache_write(kv, self.kv_a_norm_w, self.eps, pos, self.cos_sin, m.rope_interleave,
                                   ctx.slot_mapping, latent)
        mla_ops.index_k_write(k_idx, self.idx_k_ln_w, self.idx_k_ln_b, 1e-6, pos, self.cos_sin, m.rope_interleave,
                              ctx.slot_mapping, idx_k, idx_s)
        # indexer top-k
        iq = self.idx_q(q_lat).view(T, m.index_n_heads, m.index_head_dim)
        q8, wq = mla_ops.index_q_prep(iq, pos, self.cos_sin, m.rope_interleave, w_idx, self.idx_wscale)
        indices, counts = mla_ops.indexer_topk(q8, wq, idx_k, idx_s, ctx.ctx_lens, ctx.token_seq, ctx.block_table, 64,
                                               m.index_topk, ctx.max_ctx, ctx.scores_buf)
        o = self._heads(q_lat, pos, indices, counts, latent, self.h0, self.H)
        if self.full_heads:  # this rank's head slice of the whole o_proj, summed over the group
            return comm.gemm_all_reduce(o, self.o_proj.weight[:, self.h0 * self.dv:(self.h0 + self.H) * self.dv])
        return self.o_proj.forward_reduced(o)

    def _heads(self, q_lat, pos, indices, counts, latent, h0: int, H: int) -> torch.Tensor:
        """Heads [h0, h0 + H) of the queries q_lat [n, q_lora]: q_b, RoPE, W_UK absorb, latent attention
        over the selected rows, W_UV up-projection -> the o_proj input [n, H * dv]."""
        m, kvl, dr, dn = self.m, self.kvl, self.dr, self.dn
        n = q_lat.shape[0]
        if self.full_heads:  # the heads' rows of the whole q_b
            q = ops.gemm(q_lat, self.q_b.weight[h0 * (dn + dr):(h0 + H) * (dn + dr)]).view(n, H, dn + dr)
        else:
            q = self.q_b(q_lat).view(n, H, dn + dr)
        qf = torch.empty(n, H, kvl + dr, dtype=torch.bfloat16, device=q_lat.device)
        # rope part rotated straight into the query rows; absorbed nope part: per head q_nope W_UK
        # (tcgen05 batched GEMM writing the first kvl dims of the same rows)
        mla_ops.rope_into(q, pos, self.cos_sin, dn, dr, m.rope_interleave, qf, kvl)
        ops.bmm(q[:, :, :dn].transpose(0, 1), self.w_uk_t[h0:h0 + H], out=qf[:, :, :kvl].transpose(0, 1))
        o_lat = mla_ops.sparse_attention(qf, latent, indices, counts, self.sm_scale)
        # per-head up-projection W_UV, written head-interleaved as the o_proj input [n, H * dv]
        o = torch.empty(n, H * self.dv, dtype=torch.bfloat16, device=q_lat.device)
        ops.bmm(o_lat.transpose(0, 1), self.w_uv_t[h0:h0 + H], out=o.view(n, H, self.dv).transpose(0, 1))
        return o

    def forward_dp(self, x: torch.Tensor, ctx: StepContext, layer_idx: int, sp) -> torch.Tensor:
        """Data-parallel attention of the sequence-parallel layout: x [T, hidden] all tokens (gathered);
        every rank writes all tokens' cache rows (the caches stay replicated) and attends its own tokens
        [rank Tr, (rank + 1) Tr) with all heads.  Returns the o_proj output of those tokens [Tr, hidden],
        complete (no collective)."""
        latent, idx_k, idx_s = ctx.mla_caches[layer_idx]
        m = self.m
        proj = self.in_proj(x)
        ql, kvl, dr = self.ql, self.kvl, self.dr
        kv = proj[:, ql: ql + kvl + dr]
        k_idx = proj[:, ql + kvl + dr: ql + kvl + dr + m.index_head_dim]
        pos = ctx.positions
        mla_ops.latent_cache_write(kv, self.kv_a_norm_w, self.eps, pos, self.cos_sin, m.rope_interleave,
                                   ctx.slot_mapping, latent)
        mla_ops.index_k_write(k_idx, self.idx_k_ln_w, self.idx_k_ln_b, 1e-6, pos, self.cos_sin, m.rope_interleave,
                              ctx.slot_mapping, idx_k, idx_s)
        loc = slice(sp.rank * sp.Tr, (sp.rank + 1) * sp.Tr)
        Tr = sp.Tr
        q_lat = self.q_a_norm(proj[loc, :ql])  # the norm reads the strided rows
        w_idx = proj[loc, ql + kvl + dr + m.index_head_dim:]
        pos_l = pos[loc]
        iq = self.idx_q(q_lat).view(Tr, m.index_n_heads, m.index_head_dim)
        q8, wq = mla_ops.index_q_prep(iq, pos_l, self.cos_sin, m.rope_interleave, w_idx, self.idx_wscale)
        indices, counts = mla_ops.indexer_topk(q8, wq, idx_k, idx_s, ctx.ctx_lens[loc], ctx.token_seq[loc],
                                               ctx.block_table, 64, m.index_topk, ctx.max_ctx, ctx.scores_buf)
        o = self._heads(q_lat, pos_l, indices, counts, latent, 0, self.H_all)
        return ops.gemm(o, self.o_proj.weight)


# ============================================================================ MLPs
class DenseMLP(nn.Module):
    def __init__(self, hid: int, inter: int, wi: WeightInit, tp: int, tp_rank: int, limit: float = 0.0):
        super().__init__()
        g = wi.normal((inter, hid), default_std(hid), (0, tp_rank, tp))
        u = wi.normal((inter, hid), default_std(hid), (0, tp_rank, tp))
        self.gate_up = Linear(torch.cat([g, u], dim=0).contiguous())
        self.down = Linear(wi.normal((hid, inter), default_std(inter), (1, tp_rank, tp)))
        self.limit = limit

    def forward(self, x: torch.Tensor, reduce: bool = False) -> torch.Tensor:
        h = ops.silu_mul(self.gate_up(x), self.limit)
        return self.down.forward_reduced(h) if reduce else self.down(h)


def random_exl3_experts(E: int, hid: int, inter_local: int, bits_x2: int, codebook: int, wi: WeightInit,
                        tp: int, tp_rank: int, limit: float) -> moe_ops.Exl3Experts:
    """Random-init EXL3 experts (every 16-bit state is a valid code; suh = +-1,
    svh = +-1/sqrt(K))."""
    dev = wi.device
    S = 8 * bits_x2
    if wi.mode == "sliced":
        inter = inter_local * tp
        mats = {w: [] for w in ("gate", "up", "down")}
        g = torch.Generator().manual_seed(wi.seed * 31 + 17)
        for _ in range(E):
            mats["gate"].append(fx.random_matrix(hid, inter, bits_x2, codebook, generator=g))
            mats["up"].append(fx.random_matrix(hid, inter, bits_x2, codebook, generator=g))
            mats["down"].append(fx.random_matrix(inter, hid, bits_x2, codebook, generator=g))
        sl = slice(tp_rank * inter_local, (tp_rank + 1) * inter_local)
        tsl = slice(tp_rank * inter_local // 16, (tp_rank + 1) * inter_local // 16)

        def cut(m, which):
            if which == "down":
                return fx.Exl3Matrix(m.trellis[tsl].contiguous(), m.suh[sl].contiguous(), m.svh, bits_x2, codebook,
                                     inter_local, hid)
            return fx.Exl3Matrix(m.trellis[:, tsl].contiguous(), m.suh, m.svh[sl].contiguous(), bits_x2, codebook, hid,
                                 inter_local)

        ex = moe_ops.Exl3Experts.from_matrices([cut(m, "gate") for m in mats["gate"]],
                                               [cut(m, "up") for m in mats["up"]],
                                               [cut(m, "down") for m in mats["down"]], swiglu_limit=limit)
        return ex.to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(wi.seed * 7 + 1000 * pstate.get().rank + 3)

    def trellis(k, n):
        return torch.randint(-32768, 32768, (E, k // 16, n // 16, S), dtype=torch.int16, device=dev, generator=gen)

    def signs(n, scale):
        return ((torch.randint(0, 2, (E, n), device=dev, generator=gen) * 2 - 1) * scale).to(torch.float16)

    return moe_ops.Exl3Experts(
        gate_trellis=trellis(hid, inter_local), up_trellis=trellis(hid, inter_local),
        down_trellis=trellis(inter_local, hid), gate_suh=signs(hid, 1.0), up_suh=signs(hid, 1.0),
        down_suh=signs(inter_local, 1.0), gate_svh=signs(inter_local, hid ** -0.5),
        up_svh=signs(inter_local, hid ** -0.5), down_svh=signs(hid, (inter_local * tp) ** -0.5), bits_x2=bits_x2,
        codebook=codebook, hidden=hid, intermediate=inter_local, swiglu_limit=limit)


class BF16Experts(nn.Module):
    """Unquantised experts (tests / small models): per-expert loop on the GPU GEMM."""

    def __init__(self, E: int, hid: int, inter_local: int, wi: WeightInit, tp: int, tp_rank: int, limit: float):
        super().__init__()
        self.gate_up = nn.Parameter(torch.stack([torch.cat([
            wi.normal((inter_local * tp, hid), default_std(hid), (0, tp_rank, tp)),
            wi.normal((inter_local * tp, hid), default_std(hid), (0, tp_rank, tp))]) for _ in range(E)]),
            requires_grad=False)
        self.down = nn.Parameter(torch.stack([wi.normal((hid, inter_local * tp), default_std(inter_local * tp),
                                                        (1, tp_rank, tp)) for _ in range(E)]), requires_grad=False)
        self.limit = limit

    expert_map = None  # global expert -> local index (-1: not on this rank), expert parallel only

    def forward(self, x, ids, w, add=None, reduce: bool = False):
        out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
        for e in range(self.gate_up.shape[0]):
            ge = e if self.expert_map is None else int((self.expert_map == e).nonzero()[0, 0])
            mask = ids == ge  # masked ids (-1, experts of other ranks) match no expert
            rows = mask.any(-1).nonzero()[:, 0]
            if rows.numel() == 0:
                continue
            h = ops.silu_mul(ops.gemm(x[rows], self.gate_up[e]), self.limit)
            y = ops.gemm(h, self.down[e]).float()
            out[rows] += (w * mask).sum(-1)[rows, None] * y
        if add is not None:
            out += add.float()
        out = out.to(x.dtype)
        return comm.tp_all_reduce(out) if reduce else out


class MoE(nn.Module):
    """Router, routed experts and shared expert.  Routed experts are split across the TP group
    either by intermediate columns (every rank holds a slice of every expert; whole H128 blocks for
    EXL3, vllm_sm80/kernels/exl3/quant.py:869) or, with expert parallelism, whole (rank r holds
    experts [r E/tp, (r+1) E/tp)).  Tokens are replicated over the group (tensor-parallel
    attention), so the expert-parallel dispatch is the local selection of the assignments whose
    expert this rank holds (``expert_map``), and the combine of every rank's partial output is the
    fused combine + all-reduce -- the reference's EP layout, which dispatches by all-gather and
    combines by reduce-scatter (vllm_sm80/kernels/exl3/quant.py:1913-1934)."""

    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        mc = cfg.moe
        self.mc = mc
        hid = cfg.hidden_size
        ep = pstate.get().expert_parallel and tp > 1
        self.gate = Linear(wi.normal((mc.num_experts, hid), default_std(hid)))
        # router logits precision (the reference's `moe_router_dtype` switch): fp32 from the GEMM, or
        # rounded to bf16 by the GEMM's epilogue (the top-k reads them as fp32 either way)
        self.router_out = torch.float32 if mc.router_dtype == "float32" else torch.bfloat16
        self.e_bias = None
        if mc.router != "softmax":
            self.e_bias = nn.Parameter(wi.uniform((mc.num_experts,), -0.05, 0.05), requires_grad=False)
        if ep:
            assert mc.num_experts % tp == 0, "expert parallel needs the experts to divide over the group"
            e_local = mc.num_experts // tp
            first = tp_rank * e_local
            emap = torch.full((mc.num_experts,), -1, dtype=torch.int32)
            emap[first:first + e_local] = torch.arange(e_local, dtype=torch.int32)
            self.experts = self._experts(mc, hid, mc.intermediate, wi, 1, 0, first, e_local)
            self.experts.expert_map = emap.to(wi.device)
        else:
            assert mc.intermediate % tp == 0
            self.experts = self._experts(mc, hid, mc.intermediate // tp, wi, tp, tp_rank, 0, mc.num_experts)
        self.shared = None
        # with expert parallelism the shared expert is replicated (whole on every rank): the
        # sequence-parallel layout runs it on each rank's own tokens; steps on the all-reduce path let
        # rank 0 add it
        self.shared_replicated = ep
        if mc.num_shared:
            st_tp, st_rank = (1, 0) if ep else (tp, tp_rank)
            self.shared = DenseMLP(hid, mc.shared_intermediate * mc.num_shared, wi, st_tp, st_rank, mc.swiglu_limit)

    @staticmethod
    def _experts(mc, hid, inter_local, wi, tp, tp_rank, first: int, count: int):
        """`count` experts starting at global expert `first` (`sliced` init draws every expert and
        keeps these, so a model is the same under any split)."""
        E = mc.num_experts
        subset = not (first == 0 and count == E)
        n_draw = E if (subset and wi.mode == "sliced") else count
        if mc.expert_format == "exl3":
            assert inter_local % 128 == 0, "EXL3 TP cuts must keep whole H128 blocks"
            ex = random_exl3_experts(n_draw, hid, inter_local, mc.exl3_bits_x2, mc.exl3_codebook, wi, tp, tp_rank,
                                     mc.swiglu_limit)
            if n_draw != count:
                ex = ex.select(first, count)
            return ex
        if mc.expert_format == "bf16":
            ex = BF16Experts(n_draw, hid, inter_local, wi, tp, tp_rank, mc.swiglu_limit)
            if n_draw != count:
                ex.gate_up = nn.Parameter(ex.gate_up[first:first + count].contiguous(), requires_grad=False)
                ex.down = nn.Parameter(ex.down[first:first + count].contiguous(), requires_grad=False)
            return ex
        from . import marlin_experts

        ex = marlin_experts.random_marlin_experts(n_draw, hid, inter_local, wi, tp, tp_rank)
        if n_draw != count:
            ex = ex.select(first, count)
        return ex

    _aux_streams: dict = {}

    def _aux_stream(self, dev) -> torch.cuda.Stream:
        s = MoE._aux_streams.get(dev)
        if s is None:
            s = MoE._aux_streams[dev] = torch.cuda.Stream(dev)
        return s

    def forward(self, x: torch.Tensor, reduce: bool = False) -> torch.Tensor:
        """reduce: return the output summed over the tensor-parallel group."""
        logits = self.gate(x, out_dtype=self.router_out)
        ids, w = moe_ops.topk(logits, self.mc.top_k, self.mc.router_mode, self.e_bias, self.mc.routed_scaling,
                              self.mc.renormalize)
        shared = None
        need_shared = self.shared is not None and not (self.shared_replicated and reduce and pstate.get().tp_rank != 0)
        if need_shared and x.is_cuda and isinstance(self.experts, moe_ops.Exl3Experts) and _shared_stream_on():
            # the shared expert on a second stream while this one builds the assignments, rotates the
            # inputs and runs the routed experts; joined before the combine adds it (the reference's
            # shared-expert aux-stream reorder, vllm_sm80/layers/moe/shared_experts.py:67).  Works under
            # CUDA-graph capture (fork / join of the capturing stream).
            cur = torch.cuda.current_stream(x.device)
            aux = self._aux_stream(x.device)
            aux.wait_stream(cur)
            with torch.cuda.stream(aux):
                shared = self.shared(x)
            x.record_stream(aux)
            y, slot_of, sw = moe_ops.exl3_moe_rows(x, ids, w, self.experts)
            cur.wait_stream(aux)
            shared.record_stream(cur)
            return moe_ops.exl3_combine(y, slot_of, sw, ids.shape[1], shared, x.shape[0], x.shape[1], reduce)
        if need_shared:
            shared = self.shared(x)
        if isinstance(self.experts, moe_ops.Exl3Experts):
            return moe_ops.exl3_moe(x, ids, w, self.experts, add=shared, reduce=reduce)
        from ..ops.dequant import MarlinExperts, marlin_moe

        if isinstance(self.experts, MarlinExperts):
            return marlin_moe(x, ids, w, self.experts, add=shared, reduce=reduce)
        return self.experts(x, ids, w, add=shared, reduce=reduce)


    def forward_sp(self, h: torch.Tensor, sp) -> torch.Tensor | None:
        """Sequence-parallel form (expert parallel): h [Tr, H] this rank's tokens.  Routes them, sends each
        row to the ranks holding its experts, runs this rank's experts on the rows it received and sends
        the weighted sums back to the owners (summed by the next residual norm).  Returns the shared
        expert's output of the local tokens (added by that norm) or None."""
        mc = self.mc
        logits = self.gate(h, out_dtype=self.router_out).float()
        sp.route_dispatch(logits, h, mc.top_k, mc.router_mode, self.e_bias, mc.routed_scaling, mc.renormalize,
                          mc.num_experts // sp.world)
        # the shared expert runs while the dispatched rows travel
        shared = self.shared(h) if self.shared is not None else None
        x_r, ids_r, w_r = sp.dispatch_recv()
        if sp.fused and isinstance(self.experts, moe_ops.Exl3Experts):
            y, slot_of, sw = moe_ops.exl3_moe_rows(x_r, ids_r, w_r, self.experts, build=sp.build_assignments)
            sp.combine_push(y, slot_of, sw, mc.top_k)
            return shared
        if isinstance(self.experts, moe_ops.Exl3Experts):
            partial = moe_ops.exl3_moe(x_r, ids_r, w_r, self.experts, out_f32=True)
        else:
            from ..ops.dequant import MarlinExperts, marlin_moe

            if isinstance(self.experts, MarlinExperts):
                partial = marlin_moe(x_r, ids_r, w_r, self.experts, out_f32=True)
            else:
                partial = self.experts(x_r, ids_r, w_r)
        sp.combine_partial(partial)
        return shared


# ============================================================================ model
def _shared_stream_on() -> bool:
    from .. import envs

    return bool(envs.get("VLLM_B200_SHARED_EXPERT_STREAM"))


class HyperConnection(nn.Module):
    """Coefficient parameters of one mHC boundary: fn [2n + n^2, n d], scale [3], base [2n + n^2]
    (fp32, replicated over tensor-parallel ranks)."""

    def __init__(self, cfg: ModelConfig, wi: WeightInit):
        super().__init__()
        n, d = cfg.hc_mult, cfg.hidden_size
        N = 2 * n + n * n
        self.fn = nn.Parameter(wi.normal((N, n * d), (n * d) ** -0.5, dtype=torch.float32), requires_grad=False)
        self.scale = nn.Parameter(wi.uniform((3,), 0.5, 1.5).float(), requires_grad=False)
        self.base = nn.Parameter(wi.uniform((N,), -0.5, 0.5).float(), requires_grad=False)

    def __call__(self, state: "HCState", norm: RMSNorm, cfg: ModelConfig) -> tuple["HCState", torch.Tensor]:
        H, inp, post, comb, pre = mhc_ops.post_pre(
            state.x, state.H, state.post, state.comb, self.fn, self.scale, self.base, norm.weight,
            rms_eps=cfg.rms_eps, eps=cfg.hc_eps, post_mult=cfg.hc_post_mult, iters=cfg.hc_sinkhorn_iters,
            norm_eps=norm.eps, delayed=cfg.hc_delayed, pre_mix=state.pre_mix)
        return HCState(None, H, post, comb, pre if cfg.hc_delayed else None), inp


def hc_hop_fields(cfg: ModelConfig, T: int) -> list[tuple[str, tuple[int, ...], torch.dtype]]:
    """The mHC state crossing a pipeline-stage boundary after a layer: the pending sublayer output,
    the streams, the post / comb it is applied with and (delayed form) the carried pre."""
    n, d = cfg.hc_mult, cfg.hidden_size
    f = [("x", (T, d), torch.bfloat16), ("H", (T, n, d), torch.bfloat16), ("post", (T, n), torch.float32),
         ("comb", (T, n, n), torch.float32)]
    if cfg.hc_delayed:
        f.append(("pre_mix", (T, n), torch.float32))
    return f


def _hop_segments(cfg: ModelConfig, T: int):
    off, segs = 0, []
    for name, shape, dt in hc_hop_fields(cfg, T):
        nb = math.prod(shape) * torch.empty((), dtype=dt).element_size()
        segs.append((name, shape, dt, off, nb))
        off += (nb + 15) // 16 * 16  # every segment 16-byte aligned
    return segs, off


def hc_hop_bytes(cfg: ModelConfig, T: int) -> int:
    return _hop_segments(cfg, T)[1]


def hc_pack(state: "HCState", cfg: ModelConfig) -> torch.Tensor:
    """The state as one flat uint8 buffer (one p2p message per hop; the layout follows from T)."""
    T = state.H.shape[0]
    segs, total = _hop_segments(cfg, T)
    buf = torch.empty(total, dtype=torch.uint8, device=state.H.device)
    for name, shape, dt, off, nb in segs:
        buf[off:off + nb].view(dt).view(shape).copy_(getattr(state, name))
    return buf


def hc_unpack(buf: torch.Tensor, cfg: ModelConfig, T: int) -> "HCState":
    segs, _ = _hop_segments(cfg, T)
    vals = {name: buf[off:off + nb].view(dt).view(shape) for name, shape, dt, off, nb in segs}
    return HCState(vals["x"], vals["H"], vals["post"], vals["comb"], vals.get("pre_mix"))


@dataclass
class HCState:
    """The mHC residual between sublayers: streams H [T, n, d], the pending sublayer output x with
    the post / comb it is applied with at the next boundary, and (delayed form) the carried pre."""
    x: torch.Tensor | None
    H: torch.Tensor
    post: torch.Tensor | None = None
    comb: torch.Tensor | None = None
    pre_mix: torch.Tensor | None = None


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, idx: int, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        self.idx = idx
        self.kind = cfg.layer_types[idx]
        self.input_norm = RMSNorm(wi.ones_plus(cfg.hidden_size, 0.05), cfg.rms_eps)
        self.post_norm = RMSNorm(wi.ones_plus(cfg.hidden_size, 0.05), cfg.rms_eps)
        if self.kind == "dsa":
            from .dsv4 import DSAAttention

            self.attn = DSAAttention(cfg, wi, tp, tp_rank, idx)
        elif self.kind == "gqa":
            from .qwen import GatedAttention

            self.attn = GatedAttention(cfg, wi, tp, tp_rank)
        elif self.kind == "kda" and cfg.kda.mode == "gdn":
            from .qwen import GDNAttention

            self.attn = GDNAttention(cfg, wi, tp, tp_rank)
        else:
            self.attn = (KDAAttention if self.kind == "kda" else MLAAttention)(cfg, wi, tp, tp_rank)
        self.engram = None
        if idx in cfg.engram_layers:
            from .engram import EngramBlock

            self.engram = EngramBlock(cfg, wi)
        mt = cfg.mlp_types[idx]
        if mt == "moe":
            self.mlp = MoE(cfg, wi, tp, tp_rank)
        elif mt == "dense":
            self.mlp = DenseMLP(cfg.hidden_size, cfg.dense_intermediate, wi, tp, tp_rank)
        else:
            self.mlp = None
        self.cfg = cfg
        if cfg.hc_mult:
            self.hc_attn = HyperConnection(cfg, wi)
            self.hc_mlp = HyperConnection(cfg, wi) if self.mlp is not None else None

    def forward_hc(self, state: HCState, ctx: StepContext) -> HCState:
        """mHC form: each sublayer reads the collapsed, normalised streams at its boundary and
        leaves its output pending for the next boundary's post."""
        state, h = self.hc_attn(state, self.input_norm, self.cfg)
        state.x = self.attn(h, ctx, self.idx)
        if self.engram is not None:
            self.engram.add_(state.x, h, ctx.engram_rows, ctx.engram_ready)
        if self.mlp is not None:
            # the attention output's post, then the MLP input, in one boundary op
            state, h = self.hc_mlp(state, self.post_norm, self.cfg)
            state.x = self.mlp(h, reduce=True)
        return state

    def forward_sp(self, sp, residual: torch.Tensor, pending: tuple, ctx: StepContext) -> tuple:
        """Sequence-parallel layer (the step's tokens sharded over the group, parallel/sp.py).
        `pending` is how the layer input reaches this rank's residual rows: ("local", x) for the
        embeddings, ("rs", None) for a reduce-scattered projection, ("comb", shared_out) for a combined
        MoE output, ("add", a) for rows computed on this rank.  Returns the pending form of this
        layer's output."""
        sp.apply(pending, residual, self.input_norm.weight, self.input_norm.eps, ag=True)
        if isinstance(self.attn, MLAAttention) and self.attn.full_heads:
            # data-parallel attention: this rank's tokens, all heads, output complete on this rank.  In
            # the scope, its input GEMM is the all-gather area's first reader and waits for the peers'
            # rows (it issues no row-parallel reduction)
            with sp_scope(sp):
                a = self.attn.forward_dp(sp.gathered(), ctx, self.idx, sp)
            if self.mlp is None:
                return ("add", a)
            h = torch.empty_like(residual)
            sp.norm("add", residual, self.post_norm.weight, self.post_norm.eps, x=a, out=h,
                    ag=not isinstance(self.mlp, MoE))
            return self._mlp_sp(sp, residual, h)
        with sp_scope(sp):
            # the attention's first read of the gathered rows is its input GEMM, which waits for the
            # all-gather itself when it is a bf16 projection; otherwise wait before the attention
            first = getattr(self.attn, "in_proj", None) or getattr(self.attn, "wq_a", None)
            self.attn(sp.gathered(wait=not isinstance(first, Linear)), ctx, self.idx)
        if self.mlp is None:
            return ("rs", None)
        h = torch.empty_like(residual)
        sp.norm("rs", residual, self.post_norm.weight, self.post_norm.eps, out=h, ag=not isinstance(self.mlp, MoE))
        return self._mlp_sp(sp, residual, h)

    def _mlp_sp(self, sp, residual: torch.Tensor, h: torch.Tensor) -> tuple:
        """The MLP half of a sequence-parallel layer; h [Tr, hidden] the post-attention norm of this
        rank's tokens (also all-gathered when the MLP is a dense tensor-parallel one)."""
        if isinstance(self.mlp, MoE):
            return ("comb", self.mlp.forward_sp(h, sp))
        # dense MLP, tensor parallel: all-gather in (pushed by the norm), reduce-scatter out
        with sp_scope(sp):
            self.mlp(sp.gathered(), reduce=True)
        return ("rs", None)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None, ctx: StepContext):
        if residual is None:
            residual = x
            h = self.input_norm(x)
        else:
            h = self.input_norm(x, residual)
        a = self.attn(h, ctx, self.idx)  # row-parallel o_proj: already summed over the TP group
        if self.engram is not None:
            self.engram.add_(a, h, ctx.engram_rows, ctx.engram_ready)
        if self.mlp is None:  # the next layer's fused norm adds the attention output
            return a, residual
        h = self.post_norm(a, residual)
        return self.mlp(h, reduce=True), residual


def stage_layers(num_layers: int, pp_size: int, pp_rank: int) -> tuple[int, int]:
    """Layers [start, end) of pipeline stage `pp_rank` (contiguous, sizes differ by at most one)."""
    base, extra = divmod(num_layers, pp_size)
    start = pp_rank * base + min(pp_rank, extra)
    return start, start + base + (1 if pp_rank < extra else 0)


class HybridForCausalLM(nn.Module):
    """The decoder stack of one pipeline stage (all of it without pipeline parallelism).

    Stage 0 embeds the tokens; a later stage takes the previous stage's (hidden, residual) pair;
    the last stage applies the final norm and holds the vocab-parallel LM head.  The last stage
    also keeps the embedding (the MTP head reads it).  With `sliced` init every layer is drawn
    and the stage keeps its own, so a model is the same under any split."""

    def __init__(self, cfg: ModelConfig, device="cuda", seed: int = 0, init_mode: str = "local"):
        super().__init__()
        st = pstate.get()
        tp, tp_rank = st.tp_size, st.tp_rank
        self.cfg = cfg
        wi = WeightInit(seed, device, init_mode)
        self.init_mode = init_mode
        self.first, self.last = st.is_first_pp, st.is_last_pp
        self.layer_start, self.layer_end = stage_layers(cfg.num_layers, st.pp_size, st.pp_rank)
        embed = wi.normal((cfg.vocab_size, cfg.hidden_size), 1.0) if (self.first or self.last or
                                                                      init_mode == "sliced") else None
        self.embed = nn.Parameter(embed, requires_grad=False) if (self.first or self.last) else None
        layers = []
        for i in range(cfg.num_layers):
            local = self.layer_start <= i < self.layer_end
            if local or init_mode == "sliced":
                layer = DecoderLayer(cfg, i, wi, tp, tp_rank)
                if local:
                    layers.append(layer)
        self.layers = nn.ModuleList(layers)
        norm_w = wi.ones_plus(cfg.hidden_size, 0.05)
        assert cfg.vocab_size % tp == 0
        self.vocab_local = cfg.vocab_size // tp
        self.vocab_offset = tp_rank * self.vocab_local
        head = wi.normal((cfg.vocab_size, cfg.hidden_size), default_std(cfg.hidden_size), (0, tp_rank, tp)) \
            if (self.last or init_mode == "sliced") else None
        self.norm = RMSNorm(norm_w, cfg.rms_eps) if self.last else None
        self.lm_head = Linear(head) if self.last else None
        # layers whose output the forward keeps in `aux_hidden` (set by a DFlash drafter)
        self.aux_layer_ids: tuple[int, ...] = ()
        self.aux_hidden: list[torch.Tensor] = []
        # n-gram (PLE) embeddings added to the token embedding on the first stage
        self.ple = None
        if cfg.ple_heads and self.first:
            from .qwen import NgramEmbedding

            self.ple = NgramEmbedding(cfg, wi, device, seed)
        # the Engram memory table (one lookup per step serves this stage's Engram layers)
        self.engram = None
        if any(self.layer_start <= i < self.layer_end for i in cfg.engram_layers):
            from .engram import EngramMemory

            self.engram = EngramMemory(cfg, device, seed)
        self.hc_head = None
        if cfg.hc_mult and (self.last or init_mode == "sliced"):
            # the final boundary: the last sublayer's post, then the head collapse + final norm
            hc_head = HyperConnection(cfg, wi)
            self.hc_head = hc_head if self.last else None

    def forward(self, input_ids: torch.Tensor, ctx: StepContext,
                hidden_in: "tuple[torch.Tensor, torch.Tensor] | HCState | None" = None):
        """First stage: token ids; later stages: `hidden_in` = the previous stage's (hidden, residual),
        or its `HCState` with hyper-connections.  Returns the normed final hidden on the last stage,
        else what the next stage takes as `hidden_in`."""
        if self.engram is not None:
            # the lookup runs on a side stream beside the layers before the first Engram layer
            ctx.engram_rows, ctx.engram_ready = self.engram.prefetch(ctx.engram_ids)
        if self.cfg.hc_mult:
            if self.first:
                e = self.embed[input_ids]
                state = HCState(None, e.unsqueeze(1).repeat(1, self.cfg.hc_mult, 1).contiguous())
            else:
                state = hidden_in
            for layer in self.layers:
                state = layer.forward_hc(state, ctx)
            if not self.last:
                return state
            return self.hc_head(state, self.norm, self.cfg)[1]
        sp = comm.sp_for(input_ids.shape[0], self) if self.first and self.last else None
        if sp is not None:
            return self._forward_sp(input_ids, ctx, sp)
        if self.first:
            x, residual = self.embed[input_ids], None
            if self.ple is not None:
                x = x + self.ple(ctx.ple_ids)
        else:
            x, residual = hidden_in
        aux = self.aux_layer_ids
        if aux:
            self.aux_hidden = []
        for layer in self.layers:
            x, residual = layer(x, residual, ctx)
            if layer.idx in aux:  # the residual stream after this layer (a block drafter's input)
                self.aux_hidden.append(x + residual)
        if self.last:
            return self.norm(x, residual)
        return x, residual

    def supports_sp(self) -> bool:
        """Whether the sequence-parallel layout covers this model: one pipeline stage, no
        hyper-connections, no auxiliary hidden states (block drafter), MoE layers (or dense MLPs)."""
        return (self.first and self.last and not self.cfg.hc_mult and not self.aux_layer_ids and self.ple is None
                and self.engram is None
                and all(t in ("kda", "mla", "dsa") for t in self.cfg.layer_types)
                and any(isinstance(layer.mlp, MoE) for layer in self.layers))

    def _forward_sp(self, input_ids: torch.Tensor, ctx: StepContext, sp) -> torch.Tensor:
        """The whole stack with the step's tokens sharded over the tensor-parallel group; returns the
        final normed hidden states of all T tokens (all-gathered for the vocab-parallel head)."""
        T = input_ids.shape[0]
        Tr = sp.begin(T)
        x = self.embed[sp.local_slice(input_ids)]
        residual = torch.empty(Tr, self.cfg.hidden_size, dtype=torch.bfloat16, device=x.device)
        pending = ("local", x)
        for layer in self.layers:
            pending = layer.forward_sp(sp, residual, pending, ctx)
        sp.apply(pending, residual, self.norm.weight, self.norm.eps, ag=True)
        return sp.gathered(wait=True)

    def kda_recover(self, ctx: StepContext, keep: torch.Tensor) -> None:
        """After a speculative verify step: advance every verified sequence's KDA state and conv
        window over its first keep[s] tokens (the last committed token plus the accepted drafts)."""
        for layer_idx, records in ctx.kda_records.items():
            rec_state, conv = ctx.kda_states[layer_idx]
            kda_ops.kda_recover(records, keep, rec_state, conv)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """This rank's vocab shard of the logits [rows, V / tp] (bf16)."""
        return self.lm_head(hidden)

    # ------------------------------------------------------------------ cache geometry
    def kda_state_shapes(self):
        st = pstate.get()
        H = self.cfg.kda.num_heads // st.tp_size
        return (H, 128, 128), (3 * H * 128, 3)

    def kda_layer_ids(self):
        """KDA layers of this stage (global indices)."""
        return [i for i, t in enumerate(self.cfg.layer_types) if t == "kda" and self.layer_start <= i < self.layer_end]

    def mla_layer_ids(self):
        """Sparse-MLA layers of this stage (global indices)."""
        return [i for i, t in enumerate(self.cfg.layer_types) if t == "mla" and self.layer_start <= i < self.layer_end]

    def gqa_layer_ids(self):
        """Gated grouped-query attention layers of this stage (global indices)."""
        return [i for i, t in enumerate(self.cfg.layer_types) if t == "gqa" and self.layer_start <= i < self.layer_end]

    def gqa_kv_heads(self) -> int:
        """Key-value heads of this rank in a gated grouped-query attention layer."""
        g, tp = self.cfg.gqa, pstate.get().tp_size
        return g.num_kv_heads // tp if g.num_kv_heads % tp == 0 else 1

    def dsa_layer_ids(self):
        """DeepSeek-V4.1 attention layers of this stage (global indices)."""
        return [i for i, t in enumerate(self.cfg.layer_types) if t == "dsa" and self.layer_start <= i < self.layer_end]

    def layer(self, idx: int) -> "DecoderLayer":
        return self.layers[idx - self.layer_start]
