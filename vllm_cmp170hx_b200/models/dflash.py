"""DFlash block drafter: k draft tokens from one non-causal forward over a block of k + 1 queries.

On the GPU the block attention runs on the package's tcgen05 block-sparse attention kernel: each draft
layer keeps one 512-wide row per (position, key-value head), ``[k | v | 0]``, and a query row of the
block (per key-value head, its query heads in one tile) attends to the row list [its request's context
rows | the block's own rows], written into scratch rows of the same buffer; only the output half that
holds v is computed (ops/mla.py ``only_half``).  On the CPU the same attention is evaluated densely.

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


class DFlashCache:
    """One draft layer's context keys / values.  CUDA: rows [(slots + scratch) * nkv, 512] bf16 =
    [k | v | 0] per (slot, key-value head), the scratch slots after the paged ones holding a forward's
    block rows; CPU: k, v [slots, nkv, hd]."""

    def __init__(self, slots: int, nkv: int, hd: int, device, scratch: int = 0):
        self.nkv, self.hd = nkv, hd
        self.fused = torch.device(device).type == "cuda"
        if self.fused:
            if not (hd <= 128 or hd == 256):
                raise ValueError(f"DFlash head_dim {hd}: v must sit inside one 256-wide half of the rows "
                                 "(head_dim <= 128 or 256)")
            self.rows = torch.zeros((slots + scratch) * nkv, 512, dtype=torch.bfloat16, device=device)
            self.scratch0, self.scratch = slots, scratch
        else:
            self.k = torch.zeros(slots, nkv, hd, dtype=torch.bfloat16, device=device)
            self.v = torch.zeros(slots, nkv, hd, dtype=torch.bfloat16, device=device)

    def write(self, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        if self.fused:
            r = self.rows.view(-1, self.nkv, 512)
            r[slots, :, :self.hd] = k.to(r.dtype)
            r[slots, :, self.hd:2 * self.hd] = v.to(r.dtype)
        else:
            self.k[slots] = k
            self.v[slots] = v


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
        # RoPE table of the GPU path (NeoX rotate-half over the whole head)
        self.register_buffer("cos_sin", None, persistent=False)
        self.max_position = 1 << 17

    def _table(self, device) -> torch.Tensor:
        if self.cos_sin is None:
            from ..oracle.mla import rope_cos_sin

            self.cos_sin = rope_cos_sin(self.max_position, self.hd, self.theta, device)
        return self.cos_sin

    def _rope(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            return _rope(x, positions, self.theta)
        from ..ops import mla as mla_ops

        return mla_ops.rope_(x.contiguous(), positions.to(torch.int32), self._table(x.device), 0, self.hd, False)

    def kv_rows(self, h: torch.Tensor, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Key / value rows [n, nkv, hd] of normed states h [n, H]."""
        kv = ops.gemm(h, self.qkv.weight[self.nh * self.hd:])
        k, v = kv.view(-1, 2, self.nkv, self.hd).unbind(1)
        k = self._rope(self.k_norm(k.reshape(-1, self.hd)).view(-1, self.nkv, self.hd), positions)
        return k, v.contiguous()

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None, positions: torch.Tensor,
                cache: DFlashCache, ctx_slots: torch.Tensor, ctx_valid: torch.Tensor):
        """x [A * B, H] block rows of A requests (B = k + 1 each); ctx_slots [A, C] cache slots of the
        context positions, ctx_valid [A, C] the real ones (a prefix of each row)."""
        if residual is None:
            residual, h = x, self.input_norm(x)
        else:
            h = self.input_norm(x, residual)  # residual += x (in place), h = norm(residual)
        A, C = ctx_valid.shape
        B = x.shape[0] // A
        qkv = ops.gemm(h, self.qkv.weight)
        q, k, v = qkv.split([self.nh * self.hd, self.nkv * self.hd, self.nkv * self.hd], -1)
        qn = self.q_norm(q.reshape(-1, self.hd)).view(-1, self.nh, self.hd)
        k = self._rope(self.k_norm(k.reshape(-1, self.hd)).view(-1, self.nkv, self.hd), positions)
        v = v.reshape(-1, self.nkv, self.hd)
        if cache.fused:
            o = self._attend_kernel(qn, k, v, positions, cache, ctx_slots, ctx_valid, A, B)
        else:
            o = self._attend_dense(qn, k, v, positions, cache, ctx_slots, ctx_valid, A, B)
        a = ops.gemm(o.to(x.dtype), self.o_proj.weight)
        h = self.post_norm(a, residual)  # residual += a (in place), h = norm(residual)
        gu = ops.gemm(h, self.gate_up.weight)
        return ops.gemm(ops.silu_mul(gu), self.down.weight), residual

    def _attend_kernel(self, qn, k, v, positions, cache: DFlashCache, ctx_slots, ctx_valid, A: int, B: int):
        """The block attention on the block-sparse attention kernel: the block's k / v go to scratch rows,
        each (block row, key-value head) attends the row list [valid context rows | the block's rows]."""
        from ..ops import mla as mla_ops

        nkv, hd = self.nkv, self.hd
        G = self.nh // nkv
        dev = qn.device
        if A * B > cache.scratch:
            raise ValueError(f"DFlash block of {A * B} rows, the cache holds {cache.scratch} scratch rows")
        blk = cache.scratch0 + torch.arange(A * B, device=dev)
        cache.write(blk, k, v)
        C = ctx_slots.shape[1]
        n_valid = ctx_valid.sum(1)  # the valid context is a prefix of each row
        lst = torch.full((A, C + B), -1, dtype=torch.int64, device=dev)
        lst[:, :C] = torch.where(ctx_valid, ctx_slots.long(), -1)
        lst.scatter_(1, n_valid[:, None] + torch.arange(B, device=dev)[None], blk.view(A, B))
        j = torch.arange(nkv, device=dev)
        rows = torch.where(lst[:, None, :] >= 0, lst[:, None, :] * nkv + j[None, :, None], -1)  # [A, nkv, C+B]
        idx = rows[:, None].expand(A, B, nkv, C + B).reshape(A * B * nkv, C + B).to(torch.int32).contiguous()
        counts = (n_valid + B).to(torch.int32).repeat_interleave(B * nkv)
        qpad = torch.zeros(A * B * nkv, G, 512, dtype=torch.bfloat16, device=dev)
        mla_ops.rope_into(qn.reshape(A * B * nkv, G, hd), positions.to(torch.int32).repeat_interleave(nkv),
                          self._table(dev), 0, hd, False, qpad, 0)
        half = 0 if hd <= 128 else 1
        out = mla_ops.sparse_attention(qpad, cache.rows, idx, counts, hd ** -0.5, only_half=half)
        return out[..., hd:2 * hd].reshape(A * B, self.nh * hd)

    def _attend_dense(self, qn, k, v, positions, cache: DFlashCache, ctx_slots, ctx_valid, A: int, B: int):
        sl = ctx_slots.clamp_min(0).long()
        ctx_k, ctx_v = cache.k[sl], cache.v[sl]
        q = _rope(qn, positions, self.theta)
        K = torch.cat([ctx_k, k.view(A, B, self.nkv, self.hd)], 1)  # [A, C + B, nkv, hd]
        V = torch.cat([ctx_v, v.view(A, B, self.nkv, self.hd)], 1)
        valid = torch.cat([ctx_valid, torch.ones(A, B, dtype=torch.bool, device=qn.device)], 1)
        qh = q.view(A, B, self.nh, self.hd).transpose(1, 2)  # [A, nh, B, hd]
        Kh = K.transpose(1, 2)  # [A, nkv, C + B, hd]: query head h reads key / value head h // (nh / nkv)
        Vh = V.transpose(1, 2)
        o = F.scaled_dot_product_attention(qh.float(), Kh.float(), Vh.float(), attn_mask=valid[:, None, None, :],
                                           enable_gqa=self.nh != self.nkv)
        return o.transpose(1, 2).reshape(A * B, self.nh * self.hd)


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
                      caches: list[DFlashCache]) -> None:
        """Write each layer's key / value rows of the context states at `slots` (-1: none)."""
        h = self.hidden_norm(states)
        keep = slots >= 0
        for layer, cache in zip(self.layers, caches):
            k, v = layer.kv_rows(h, positions)
            cache.write(slots[keep], k[keep], v[keep])

    # bound on the context keys / values one block forward gathers (requests are split into groups)
    gather_bytes = 256 << 20

    def forward(self, bonus: torch.Tensor, last_pos: torch.Tensor, ctx_slots: torch.Tensor, ctx_valid: torch.Tensor,
                caches: list[DFlashCache], k: int) -> torch.Tensor:
        A, C = ctx_slots.shape
        if caches and caches[0].fused:  # the attention kernel reads the rows in place: no gather, no groups
            return self._forward(bonus, last_pos, ctx_slots, ctx_valid, caches, k)
        # K and V (bf16) of the context plus the block rows, gathered once and joined once (the
        # attention reads the key / value heads in place, no per-query-head copies)
        per_req = (C + k + 1) * self.dc.num_kv_heads * self.dc.head_dim * 2 * 2 * 2
        step = max(1, self.gather_bytes // max(1, per_req))
        if A <= step:
            return self._forward(bonus, last_pos, ctx_slots, ctx_valid, caches, k)
        return torch.cat([self._forward(bonus[i:i + step], last_pos[i:i + step], ctx_slots[i:i + step],
                                        ctx_valid[i:i + step], caches, k) for i in range(0, A, step)])

    def _forward(self, bonus: torch.Tensor, last_pos: torch.Tensor, ctx_slots: torch.Tensor, ctx_valid: torch.Tensor,
                 caches: list[DFlashCache], k: int) -> torch.Tensor:
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
        for layer, cache in zip(self.layers, caches):
            x, residual = layer(x, residual, pos, cache, ctx_slots, ctx_valid)
        h = self.norm(x, residual).view(A, B, -1)
        return h[:, 1:]

    def alloc_caches(self, rows: int, device, max_block_rows: int = 0) -> list[DFlashCache]:
        """Per draft layer: the context rows of `rows` cache slots, plus (GPU) scratch rows for the largest
        block forward (requests x (k + 1))."""
        dc = self.dc
        return [DFlashCache(rows, dc.num_kv_heads, dc.head_dim, device, max_block_rows) for _ in self.layers]
