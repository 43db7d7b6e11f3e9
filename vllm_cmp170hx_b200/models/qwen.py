"""Layers of the Qwen3.8-Flash-Next-style linear / full hybrid (the reference's third served family,
README.md:32-37; model classes vllm_sm80/models/qwen4_exp/sm80_model.py:72-121, PLE embedding
exl3_ple.py:436, precision switches precision.py).  The decoder stack, MoE, MTP head, caches and
engine are the package's shared ones (models/hybrid.py); this file adds the two attention kinds and the
n-gram embedding:

* :class:`GDNAttention` (layer type "kda" with ``KDAConfig.mode == "gdn"``): the gated delta net --
  fused input GEMM [q | k | v | z | b | a], causal conv + SiLU, L2-normalised q / k, one decay per head
  ``exp(-exp(A_log) * softplus(a + dt_bias))``, ``beta = sigmoid(b)``, the delta rule, gated RMSNorm with
  ``silu(z)``, row-parallel out projection.  It runs on the KDA recurrence kernel (csrc/kda.cu,
  gate_mode 1).  When value heads outnumber query / key heads, the query / key projections and conv
  taps are stored once per value head (each value head's copy of its shared head), so the kernel keeps
  one (q, k, v) triple per head; this costs the duplicated rows of the input GEMM and nothing else.
* :class:`GatedAttention` (layer type "gqa"): per query head [q | gate], per-head q / k RMSNorm, partial
  NeoX RoPE, causal attention over a paged [k | v] cache on the block attention kernel's dense mode,
  ``o * sigmoid(gate)``, row-parallel o_proj (ops/gqa.py).
* :class:`NgramEmbedding`: per-token n-gram ids (head h hashes the last ``ple_orders[h]`` tokens with the
  table's multipliers), rows from an EXL3-coded PLE table file (storage/ple.py: host LRU cache, reads,
  GPU decode), projected to the hidden size and added to the token embedding.  A row the host failed to
  read decodes to NaN, which fails only the requests whose tokens used it (the failed-input path).
"""

from __future__ import annotations

import os
import tempfile

import numpy as np
import torch
from torch import nn

from ..config import ModelConfig
from ..ops import gqa as gqa_ops
from ..ops import kda as kda_ops
from ..oracle import mla as mla_ref
from .layers import Linear, WeightInit, default_std


class GDNAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        k = cfg.kda
        Hv, D = k.num_heads, k.head_dim
        Hk = k.num_k_heads or Hv
        assert D == 128 and Hv % tp == 0, "gated delta net: head_dim 128, value heads divide over the group"
        self.H = Hv // tp
        self.D = D
        rep = Hv // Hk
        hid = cfg.hidden_size
        sd = default_std(hid)
        # logical weights of the checkpoint's shapes, then this rank's value heads with their q / k copies
        wq = wi.normal((Hk * D, hid), sd)
        wk = wi.normal((Hk * D, hid), sd)
        wv = wi.normal((Hv * D, hid), sd, (0, tp_rank, tp))
        wz = wi.normal((Hv * D, hid), sd, (0, tp_rank, tp))
        wb = wi.normal((Hv, hid), sd, (0, tp_rank, tp))
        wa = wi.normal((Hv, hid), sd, (0, tp_rank, tp))
        heads = torch.arange(tp_rank * self.H, (tp_rank + 1) * self.H) // rep  # each local value head's q / k head
        self.kv_head = heads
        pick = (heads[:, None] * D + torch.arange(D)[None]).reshape(-1).to(wq.device)
        HD = self.H * D
        rows = 4 * HD + 2 * self.H
        pad = (-rows) % 8
        self.in_proj = Linear(torch.cat([wq[pick], wk[pick], wv, wz, wb, wa,
                                         torch.zeros(pad, hid, dtype=wq.dtype, device=wq.device)], 0).contiguous())
        conv = wi.normal((2 * Hk * D + Hv * D, 4), 0.5, None)  # checkpoint order: q | k | v channels
        cq, ck = conv[:Hk * D], conv[Hk * D:2 * Hk * D]
        cv = conv[2 * Hk * D:].view(Hv, D, 4)[tp_rank * self.H:(tp_rank + 1) * self.H].reshape(HD, 4)
        self.conv_w = nn.Parameter(torch.cat([cq[pick], ck[pick], cv], 0).contiguous(), requires_grad=False)
        self.a_log = nn.Parameter(wi.uniform((Hv,), -1.0, 1.0)[tp_rank * self.H:(tp_rank + 1) * self.H].contiguous(),
                                  requires_grad=False)
        self.dt_bias = nn.Parameter(wi.uniform((Hv,), -0.5, 0.5)[tp_rank * self.H:(tp_rank + 1) * self.H].contiguous(),
                                    requires_grad=False)
        self.norm_w = nn.Parameter(wi.ones_plus(D, 0.05), requires_grad=False)
        self.o_proj = Linear(wi.normal((hid, Hv * D), default_std(Hv * D), (1, tp_rank, tp)))

    def forward(self, x: torch.Tensor, ctx, layer_idx: int) -> torch.Tensor:
        rec, conv = ctx.kda_states[layer_idx]
        proj = self.in_proj(x)
        HD = self.H * self.D
        qkv = proj[:, :3 * HD]
        z = proj[:, 3 * HD:4 * HD]
        b = proj[:, 4 * HD:4 * HD + self.H]
        a = proj[:, 4 * HD + self.H:4 * HD + 2 * self.H]
        records = None
        if ctx.kda_verify is not None:
            records = ctx.kda_records.setdefault(layer_idx, kda_ops.KdaRecords())
        o = kda_ops.kda_forward(qkv, a, b, z, ctx.cu_seqlens, ctx.kda_slots, ctx.has_init, conv, self.conv_w, None,
                                self.a_log, self.dt_bias, 0.0, self.norm_w, rec, eps=1e-6,
                                verify=ctx.kda_verify, records=records, gate_mode=1)
        return self.o_proj.forward_reduced(o)


class GatedAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, wi: WeightInit, tp: int, tp_rank: int):
        super().__init__()
        g = cfg.gqa
        HD = g.head_dim
        nh, nkv = g.num_heads, g.num_kv_heads
        assert nh % tp == 0 and (nkv % tp == 0 or tp % nkv == 0), "gqa: heads must split over the group"
        self.nh = nh // tp
        if nkv % tp == 0:
            self.nkv, kv0 = nkv // tp, tp_rank * (nkv // tp)
        else:  # fewer key-value heads than ranks: each rank keeps the one its query heads read
            self.nkv, kv0 = 1, tp_rank // (tp // nkv)
        self.eps = cfg.rms_eps
        hid = cfg.hidden_size
        sd = default_std(hid)
        wqg = wi.normal((nh * 2 * HD, hid), sd, (0, tp_rank, tp))  # per query head [q | gate]
        wk = wi.normal((nkv * HD, hid), sd)[kv0 * HD:(kv0 + self.nkv) * HD]
        wv = wi.normal((nkv * HD, hid), sd)[kv0 * HD:(kv0 + self.nkv) * HD]
        self.in_proj = Linear(torch.cat([wqg, wk, wv], 0).contiguous())
        self.q_norm_w = nn.Parameter(wi.ones_plus(HD, 0.05), requires_grad=False)
        self.k_norm_w = nn.Parameter(wi.ones_plus(HD, 0.05), requires_grad=False)
        self.o_proj = Linear(wi.normal((hid, nh * HD), default_std(nh * HD), (1, tp_rank, tp)))
        self.register_buffer("cos_sin", mla_ref.rope_cos_sin(min(cfg.max_position, 1 << 17), g.rotary_dim,
                                                             g.rope_theta, wi.device), persistent=False)

    def cache_rows(self, num_positions: int) -> tuple[int, int]:
        """Shape of this layer's paged cache: one [k | v] row per (position, local key-value head)."""
        return num_positions * self.nkv, 2 * gqa_ops.HD

    def forward(self, x: torch.Tensor, ctx, layer_idx: int) -> torch.Tensor:
        cache = ctx.gqa_caches[layer_idx]
        T = x.shape[0]
        proj = self.in_proj(x)
        G = self.nh // self.nkv
        q = torch.empty(T * self.nkv, G, 2 * gqa_ops.HD, dtype=torch.bfloat16, device=x.device)
        gqa_ops.prep(proj, self.nh, self.nkv, self.q_norm_w, self.k_norm_w, self.eps, ctx.positions, self.cos_sin,
                     ctx.slot_mapping, q, cache)
        o = gqa_ops.attention(q, cache, ctx.ctx_lens, ctx.token_seq, ctx.block_table, self.nkv, ctx.max_ctx)
        return self.o_proj.forward_reduced(gqa_ops.gate(o, proj, self.nh))


# ---------------------------------------------------------------------------------------------- PLE
def ngram_ids(tokens: np.ndarray, positions: np.ndarray, orders: list[int], offsets: np.ndarray,
              vocab: np.ndarray, mult: np.ndarray) -> np.ndarray:
    """n-gram ids of the tokens at `positions` of one sequence (tokens = the sequence so far, at least up to
    the last position): head h, order n = orders[h], key = sum_i (tok[p - i] + 1) * mult[(h + i) % M] for
    i < n (tokens before the sequence are 0), id = offsets[h] + key % vocab[h].  Returns int64 [len, heads]."""
    P = len(positions)
    H = len(orders)
    out = np.empty((P, H), dtype=np.int64)
    M = len(mult)
    for h, n in enumerate(orders):
        key = np.zeros(P, dtype=np.int64)
        for i in range(n):
            p = positions - i
            tok = np.where(p >= 0, tokens[np.maximum(p, 0)], -1) + 1
            key = (key + (tok % vocab[h]) * (int(mult[(h + i) % M]) % int(vocab[h]))) % vocab[h]
        out[:, h] = offsets[h] + key
    return out


class NgramEmbedding(nn.Module):
    def __init__(self, cfg: ModelConfig, wi: WeightInit, device, seed: int = 0):
        super().__init__()
        from ..formats import ple as fple
        from ..storage.ple import PleTable

        path, prefix = cfg.ple_path, "ple"
        if not path:
            # synthetic runs: a random table of the configured shape, written once per process
            d = tempfile.mkdtemp(prefix="b200_ple_")
            path = os.path.join(d, "ple.safetensors")
            table = fple.random_table(cfg.ple_heads, cfg.ple_vocab, cfg.ple_dim, cfg.ple_bits, seed=seed + 4242)
            table["layer_multipliers"] = torch.tensor([0x9E3779B1, 0x85EBCA77, 0xC2B2AE3D, 0x27D4EB2F],
                                                      dtype=torch.int64)
            fple.write_table(path, prefix, table, cfg.ple_bits)
        self.table = PleTable(path, prefix, device=device)
        if self.table.heads != cfg.ple_heads or self.table.dim != cfg.ple_dim:
            raise ValueError(f"PLE table {path}: {self.table.heads} heads x {self.table.dim}, the model wants "
                             f"{cfg.ple_heads} x {cfg.ple_dim}")
        self.orders = list(cfg.ple_orders) or [2] * cfg.ple_heads
        if len(self.orders) != cfg.ple_heads:
            raise ValueError("ple_orders needs one n-gram order per PLE head")
        self.max_order = max(self.orders)
        self.heads = cfg.ple_heads
        self.offsets = np.asarray(self.table._offs_cpu, dtype=np.int64)
        self.vocab = np.asarray(self.table._vocab_cpu, dtype=np.int64)
        self.mult = np.asarray(self.table.layer_multipliers.tolist(), dtype=np.int64)
        width = cfg.ple_heads * cfg.ple_dim
        self.proj = Linear(wi.normal((cfg.hidden_size, width), default_std(width)))

    def ids_of(self, tokens, positions: np.ndarray) -> np.ndarray:
        return ngram_ids(np.asarray(tokens, dtype=np.int64), positions, self.orders, self.offsets, self.vocab,
                         self.mult)

    def reserve(self, max_tokens: int) -> None:
        """Size the lookup staging for the largest step once, before any CUDA-graph capture binds it."""
        if self.table.device.type == "cuda":
            self.table._staging(max(max_tokens, 64) * self.table.heads)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """ids int64 [T, heads] (device) -> [T, hidden] bf16 to add to the token embedding."""
        if ids.is_cuda:
            rows = self.table.lookup_async(ids, fixed=torch.cuda.is_current_stream_capturing())
        else:
            rows, _ = self.table.lookup(ids)  # host path: failed tokens come back as zero rows
        return self.proj(rows)
