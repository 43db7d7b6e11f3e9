"""DFlash block drafter: k draft tokens from one non-causal forward over a block of k + 1 queries.

The target exposes the residual stream after a few of its layers (the auxiliary hidden states);
their concatenation goes through `fc` into one context state per verified position.  Each draft
layer projects a context state (after `hidden_norm`) to a key / value row -- k_norm per head and
RoPE on the key -- kept in the layer's paged context cache on the target's blocks (same slot
mapping).  A draft is one forward of the query block [bonus token, mask x k] at positions
p + 1 .. p + 1 + k (p: the last verified position): every block row attends, without a causal
mask, to the request's context rows 0..p and to all k + 1 block rows; the normed outputs of the
k mask rows go through the target's vocab-parallel LM head and are sampled as the k drafts.

Layers are Qwen3-style (q_norm / k_norm per head, RoPE over the whole head, SwiGLU MLP), the shape
the reference's DFlash drafters use (upstream vllm/model_executor/models/qwen3_dflash.py via the
reference's vllm_sm80/spec_decode/dflash_draft.py mixin; `combine_hidden_states` = `fc`).  The
drafter is replicated on every tensor-parallel rank (it is small), so drafting needs no collective
beyond the sharded sampling.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from .. import ops
from ..config import ModelConfig
from .layers import Linear, RMSNorm, WeightInit, default_std


@dataclass
class DFlashConfig:
    num_layers: int = 1
    num_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 128
    intermediate: int = 4096
    aux_layer_ids: list[int] = field(default_factory=list)  # target layers whose output feeds fc
    mask_token_id: int = 0
    rope_theta: float = 1e6

    def resolve(self, cfg: ModelConfig) -> "DFlashConfig":
        if not self.aux_layer_ids:
            L = cfg.num_layers
            self.aux_layer_ids = sorted({1, L // 2, L - 2} & set(range(L))) or [L - 1]
        return self


def _rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half RoPE over the whole head dim of x [n, heads, hd] (fp32 math)."""
    hd = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd))
    ang = positions.float()[:, None] * inv[None]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    xf = x.float()
    a, b = xf[..., : hd // 2], xf[..., hd // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1).to(x.dtype)


class DFlashLayer(nn.Module):
    def __init__(self, H: int, dc: DFlashConfig, eps: float, wi: WeightInit):
        super().__init__()
        nh, nkv, hd = dc.num_heads, dc.num_kv_heads, dc.head_dim
        self.nh, self.nkv, self.hd, self.theta = nh, nkv, hd, dc.rope_theta
        self.input_norm = RMSNorm(wi.ones_plus(H, 0.05), eps)
        self.post_norm = RMSNorm(wi.ones_plus(H, 0.05), eps)
        self.qkv = Linear(wi.normal(((nh + 2 * nkv) * hd, H), default_std(H)))
        self.q_norm = RMSNorm(wi.ones_plus(hd, 0.05), eps)
        self.k_norm = RMSNorm(wi.ones_plus(hd, 0.05), eps)
        self.o_proj = Linear(wi.normal((H, nh * hd), default_std(nh * hd)))
        self.gate_up = Linear(wi.normal((2 * dc.intermediate, H), default_std(H)))
        self.down = Linear(wi.normal((H, dc.intermediate), default_std(dc.intermediate)))

    def kv_rows(self, h: torch.Tensor, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Key / value rows [n, nkv, hd] of normed states h [n, H]."""
        kv = ops.gemm(h, self.qkv.weight[self.nh * self.hd:])
        k, v = kv.view(-1, 2, self.nkv, self.hd).unbind(1)
        k = _rope(self.k_norm(k.reshape(-1, self.hd)).view(-1, self.nkv, self.hd), positions, self.theta)
        return k, v.contiguous()

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None, positions: torch.Tensor,
                ctx_k: torch.Tensor, ctx_v: torch.Tensor, ctx_valid: torch.Tensor):
        """x [A * B, H] block rows of A requests (B = k + 1 each); ctx_k / ctx_v [A, C, nkv, hd] with
        ctx_valid [A, C]."""
        if residual is None:
            residual, h = x, self.input_norm(x)
        else:
            h = self.input_norm(x, residual)  # residual += x (in place), h = norm(residual)
        A, C = ctx_valid.shape
        B = x.shape[0] // A
        qkv = ops.gemm(h, self.qkv.weight)
        q, k, v = qkv.split([self.nh * self.hd, self.nkv * self.hd, self.nkv * self.hd], -1)
        q = _rope(self.q_norm(q.reshape(-1, self.hd)).view(-1, self.nh, self.hd), positions, self.theta)
        k = _rope(self.k_norm(k.reshape(-1, self.hd)).view(-1, self.nkv, self.hd), positions, self.theta)
        v = v.reshape(-1, self.nkv, self.hd)
        K = torch.cat([ctx_k, k.view(A, B, self.nkv, self.hd)], 1)  # [A, C + B, nkv, hd]
        V = torch.cat([ctx_v, v.view(A, B, self.nkv, self.hd)], 1)
        valid = torch.cat([ctx_valid, torch.ones(A, B, dtype=torch.bool, device=x.device)], 1)
        qh = q.view(A, B, self.nh, self.hd).transpose(1, 2)  # [A, nh, B, hd]
        Kh = K.transpose(1, 2)  # [A, nkv, C + B, hd]: query head h reads key / value head h // (nh / nkv)
        Vh = V.transpose(1, 2)
        o = F.scaled_dot_product_attention(qh, Kh, Vh, attn_mask=valid[:, None, None, :],
                                           enable_gqa=self.nh != self.nkv)
        o = o.transpose(1, 2).reshape(A * B, self.nh * self.hd).to(x.dtype)
        a = ops.gemm(o, self.o_proj.weight)
        h = self.post_norm(a, residual)  # residual += a (in place), h = norm(residual)
        gu = ops.gemm(h, self.gate_up.weight)
        g, u = gu.chunk(2, -1)
        return ops.gemm((F.silu(g.float()) * u.float()).to(x.dtype), self.down.weight), residual


class DFlashDrafter(nn.Module):
    def __init__(self, cfg: ModelConfig, dc: DFlashConfig, target, device, seed: int = 0, init_mode: str = "local"):
        super().__init__()
        self.dc = dc.resolve(cfg)
        H = cfg.hidden_size
        wi = WeightInit(seed + 9091, device, init_mode)
        n_aux = len(self.dc.aux_layer_ids)
        self.fc = Linear(wi.normal((H, n_aux * H), default_std(n_aux * H)))
        self.hidden_norm = RMSNorm(wi.ones_plus(H, 0.05), cfg.rms_eps)
        self.layers = nn.ModuleList(DFlashLayer(H, self.dc, cfg.rms_eps, wi) for _ in range(self.dc.num_layers))
        self.norm = RMSNorm(wi.ones_plus(H, 0.05), cfg.rms_eps)
        # confidence head: the estimated acceptance of each draft position (a verify-depth feature)
        self.conf_head = Linear(wi.normal((1, H), default_std(H)))
        self.target = [target]  # embedding and LM head are the target's (not submodules)

    def confidence(self, h: torch.Tensor) -> torch.Tensor:
        """sigmoid of the confidence head over the mask rows' hidden states [A, k, H] -> [A, k]."""
        A, k, H = h.shape
        return torch.sigmoid(ops.gemm(h.reshape(A * k, H), self.conf_head.weight, out_dtype=torch.float32)).view(A, k)

    def context_states(self, aux: list[torch.Tensor]) -> torch.Tensor:
        """The target's auxiliary hidden states [n, H] each -> context states [n, H]."""
        return ops.gemm(torch.cat(aux, -1), self.fc.weight)

    def store_context(self, states: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                      caches: list[tuple[torch.Tensor, torch.Tensor]]) -> None:
        """Write each layer's key / value rows of the context states at `slots` (-1: none)."""
        h = self.hidden_norm(states)
        keep = slots >= 0
        for layer, (kc, vc) in zip(self.layers, caches):
            k, v = layer.kv_rows(h, positions)
            kc[slots[keep]] = k[keep]
            vc[slots[keep]] = v[keep]

    # bound on the context keys / values one block forward gathers (requests are split into groups)
    gather_bytes = 256 << 20

    def forward(self, bonus: torch.Tensor, last_pos: torch.Tensor, ctx_slots: torch.Tensor, ctx_valid: torch.Tensor,
                caches: list[tuple[torch.Tensor, torch.Tensor]], k: int) -> torch.Tensor:
        A, C = ctx_slots.shape
        # K and V (bf16) of the context plus the block rows, gathered once and joined once (the
        # attention reads the key / value heads in place, no per-query-head copies)
        per_req = (C + k + 1) * self.dc.num_kv_heads * self.dc.head_dim * 2 * 2 * 2
        step = max(1, self.gather_bytes // max(1, per_req))
        if A <= step:
            return self._forward(bonus, last_pos, ctx_slots, ctx_valid, caches, k)
        return torch.cat([self._forward(bonus[i:i + step], last_pos[i:i + step], ctx_slots[i:i + step],
                                        ctx_valid[i:i + step], caches, k) for i in range(0, A, step)])

    def _forward(self, bonus: torch.Tensor, last_pos: torch.Tensor, ctx_slots: torch.Tensor, ctx_valid: torch.Tensor,
                 caches: list[tuple[torch.Tensor, torch.Tensor]], k: int) -> torch.Tensor:
        """bonus [A] (the token after the last verified position), last_pos [A]; ctx_slots [A, C]
        cache slots of the context positions (ctx_valid marks the real ones).  Returns the normed
        hidden states [A, k, H] of the k mask rows."""
        t = self.target[0]
        A = bonus.shape[0]
        B = k + 1
        ids = torch.full((A, B), self.dc.mask_token_id, dtype=torch.long, device=bonus.device)
        ids[:, 0] = bonus
        pos = (last_pos[:, None] + 1 + torch.arange(B, device=bonus.device)[None]).reshape(-1)
        x = t.embed[ids.reshape(-1)]
        residual = None
        sl = ctx_slots.clamp_min(0).long()
        for layer, (kc, vc) in zip(self.layers, caches):
            x, residual = layer(x, residual, pos, kc[sl], vc[sl], ctx_valid)
        h = self.norm(x, residual).view(A, B, -1)
        return h[:, 1:]

    def alloc_caches(self, rows: int, device) -> list[tuple[torch.Tensor, torch.Tensor]]:
        dc = self.dc
        return [(torch.zeros(rows, dc.num_kv_heads, dc.head_dim, dtype=torch.bfloat16, device=device),
                 torch.zeros(rows, dc.num_kv_heads, dc.head_dim, dtype=torch.bfloat16, device=device))
                for _ in self.layers]
