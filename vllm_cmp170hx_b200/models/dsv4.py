"""DeepSeek-V4.1 attention layer (layer type "dsa") of the hybrid decoder.

Projections (the reference's layer: vllm_sm80/models/deepseek_v41/sm80_attention.py:303, projections
:682, output :851-885): q = wq_b(q_norm(wq_a(x))) per head (512 wide, RoPE on the last 64);
kv = kv_norm(wkv(x)); for a compressed layer the compressor's fp32 [kv | score] rows (ratio 2) or
the kv row itself (ratio 1), the indexer's query wq_b_index(q latent) and head weights
weights_proj(x).  The attention core (ops/dsv4_attn.py) keeps the window, compressed and index-key
caches and returns the per-head outputs (inverse RoPE and FP8 qdq applied); grouped wo_a then the
row-parallel wo_b (summed over the tensor-parallel group) give the layer output.

Heads, sinks and wo_a groups are split over tensor-parallel ranks; the indexer is replicated (it
is small) and rounds its head sums in the reference's rank groups (`index_rank_groups`), so every
rank selects the same rows.  The indexer's score width is the step's host bound on visible groups
(`StepContext.max_ctx`), so a step reads no device value on the host and decode steps run from CUDA
graphs like the other layer types.
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import ModelConfig
from ..ops.dsv4_attn import DSv4AttnCore, DSv4AttnSpec
from .layers import GroupedLinear, Linear, RMSNorm, WeightInit, default_std


def dsa_ratio(cfg: ModelConfig, idx: int) -> int:
    """Compression ratio of global layer idx (its position among the "dsa" layers)."""
    k = cfg.layer_types[:idx].count("dsa")
    r = cfg.dsa.compress_ratios
    ratio = r[k % len(r)] if r else 1
    if ratio not in (0, 1, 2):
        # the compressor, its caches and the checkpoint names exist for ratios 0 (window only), 1 and 2
        raise ValueError(f"DeepSeek-V4.1 layer {idx}: compression ratio {ratio} is not supported (0, 1 or 2)")
    return ratio


class DSAAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int, idx: int):
        super().__init__()
        a = cfg.dsa
        hid, d, ql = cfg.hidden_size, a.head_dim, a.q_lora_rank
        assert d == 512 and a.rope_dim == 64 and a.num_heads % tp == 0 and a.o_groups % tp == 0
        assert a.num_heads % a.o_groups == 0
        self.a, self.eps = a, cfg.rms_eps
        self.H = a.num_heads // tp
        self.G = a.o_groups // tp
        self.ratio = dsa_ratio(cfg, idx)
        sd = default_std(hid)
        self.wq_a = Linear(wi.normal((ql, hid), sd))
        self.q_norm = RMSNorm(wi.ones_plus(ql, 0.05), cfg.rms_eps)
        self.wq_b = Linear(wi.normal((a.num_heads * d, ql), default_std(ql), (0, tp_rank, tp)))
        self.wkv = Linear(wi.normal((d, hid), sd))
        self.kv_norm = RMSNorm(wi.ones_plus(d, 0.05), cfg.rms_eps)
        self.sink = nn.Parameter(wi.normal((a.num_heads,), 1.0, (0, tp_rank, tp), dtype=torch.float32),
                                 requires_grad=False)
        hpg = a.num_heads // a.o_groups
        self.wo_a = GroupedLinear(wi.normal((a.o_groups, a.o_lora_rank, hpg * d), default_std(hpg * d),
                                            (0, tp_rank, tp)))
        self.wo_b = Linear(wi.normal((hid, a.o_groups * a.o_lora_rank), default_std(a.o_groups * a.o_lora_rank),
                                     (1, tp_rank, tp)))
        self.comp_norm = self.wk = self.k_norm = self.wkv_c = self.idx_q = self.idx_w = None
        if self.ratio:
            self.comp_norm = nn.Parameter(wi.ones_plus(d, 0.05), requires_grad=False)
            # the compressor's own projection: [kv | gate score] (ratio 2) or kv (ratio 1)
            self.wkv_c = Linear(wi.normal(((2 if self.ratio == 2 else 1) * d, hid), sd))
            self.idx_q = Linear(wi.normal((a.index_n_heads * a.index_head_dim, ql), default_std(ql)))
            self.idx_w = Linear(wi.normal((a.index_n_heads, hid), sd))
            self.wk = nn.Parameter(wi.normal((a.index_head_dim, d), default_std(d)), requires_grad=False)
            self.k_norm = nn.Parameter(wi.ones_plus(a.index_head_dim, 0.05), requires_grad=False)
        self.register_buffer("freqs", 1.0 / (a.rope_theta ** (torch.arange(0, a.rope_dim, 2, dtype=torch.float32,
                                                                             device=wi.device) / a.rope_dim)),
                             persistent=False)

    def spec(self) -> DSv4AttnSpec:
        a = self.a
        return DSv4AttnSpec(heads=self.H, window=a.window, ratio=self.ratio, index_heads=a.index_n_heads,
                            index_dim=a.index_head_dim, index_topk=a.index_topk,
                            index_heads_per_rank=a.index_n_heads // a.index_rank_groups, out_groups=self.G,
                            eps=self.eps)

    def make_core(self, num_slots: int, group_rows: int, max_step_tokens: int, spec_width: int, device):
        """Caches for `num_slots` sequence slots; spec_width = drafts per verify step (0: none)."""
        return DSv4AttnCore(self.spec(), num_slots, group_rows, max_step_tokens, self.freqs, self.sink,
                            self.comp_norm, self.wk, self.k_norm, device, carry_rows=spec_width + 2,
                            ring_extra=spec_width)

    def forward(self, x: torch.Tensor, ctx, layer_idx: int) -> torch.Tensor:
        core = ctx.dsa_cores[layer_idx]
        T = x.shape[0]
        a = self.a
        qr = self.q_norm(self.wq_a(x))
        q = self.wq_b(qr).view(T, self.H, a.head_dim)
        kv = self.kv_norm(self.wkv(x))
        ks = None
        if self.ratio == 2:
            ks = self.wkv_c(x, out_dtype=torch.float32)
        elif self.ratio == 1:
            ks = self.wkv_c(x)  # bf16 row, normalised by the core
        iq = self.idx_q(qr).view(T, a.index_n_heads, a.index_head_dim) if self.ratio else None
        iw = self.idx_w(x) if self.ratio else None
        ng = max(1, ctx.max_ctx // self.ratio) if self.ratio else None  # host bound: no device read
        # tokens without a cache slot (the padding of a CUDA-graph batch) write no group, ring or carry row
        valid = ctx.slot_mapping >= 0 if ctx.slot_mapping is not None else None
        o = core.step(ctx.token_seq, ctx.positions, ctx.kda_slots, ctx.block_table, q, kv, ks, iq, iw, max_groups=ng,
                      valid=valid)
        y = self.wo_a(o.reshape(T, self.G, (self.H // self.G) * a.head_dim))
        return self.wo_b.forward_reduced(y)
