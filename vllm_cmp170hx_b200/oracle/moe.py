"""References of MoE routing and expert evaluation (fp32)."""

from __future__ import annotations

import torch

from ..formats import exl3 as fx


def topk(logits: torch.Tensor, k: int, mode: int, bias: torch.Tensor | None = None, scale: float = 1.0,
         renorm: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """mode 0 softmax (renormalised over the k picked), 1 sigmoid + bias-select (GLM),
    2 sqrt(softplus) + bias-select with weights s / (sum + 1e-20) (DeepSeek-V4.1,
    vllm_sm80/models/deepseek_v41/sm80_moe.py:19-26).  Ties -> lowest expert id."""
    l = logits.float()
    if mode == 0:
        s = torch.softmax(l, dim=-1)
        key = s
    elif mode == 1:
        s = torch.sigmoid(l)
        key = s + (bias.float() if bias is not None else 0)
    else:
        s = torch.sqrt(torch.nn.functional.softplus(l))
        key = s + (bias.float() if bias is not None else 0)
    E = l.shape[-1]
    # stable tie-break: sort by (-key, index)
    order = torch.argsort(-key, dim=-1, stable=True)
    ids = order[:, :k]
    w = torch.gather(s, 1, ids)
    if renorm:
        w = w / (w.sum(-1, keepdim=True) + (1e-20 if mode == 2 else 0.0))
    return ids.to(torch.int32), (w * scale).float()


def exl3_experts(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, experts: dict, swiglu_limit=None,
                 dense_cache: dict | None = None) -> torch.Tensor:
    """out[t] = sum_j w[t,j] * down_e(silu(gate_e(x)) * up_e(x)) with EXL3 matrices; fp32."""
    T, H = x.shape
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    emap = experts.get("expert_map")
    for t in range(T):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e < 0:  # an expert of another rank (masked id)
                continue
            if emap is not None:
                e = int(emap[e])
                if e < 0:
                    continue
            g = fx.linear(x[t:t + 1], experts["gate"][e], _w(dense_cache, ("g", e), experts["gate"][e]))
            u = fx.linear(x[t:t + 1], experts["up"][e], _w(dense_cache, ("u", e), experts["up"][e]))
            if swiglu_limit:
                g = g.clamp(max=swiglu_limit)
                u = u.clamp(-swiglu_limit, swiglu_limit)
            h = torch.nn.functional.silu(g) * u
            d = fx.linear(h, experts["down"][e], _w(dense_cache, ("d", e), experts["down"][e]))
            out[t] += float(weights[t, j]) * d[0]
    return out


def _w(cache, key, m):
    if cache is None:
        return None
    if key not in cache:
        cache[key] = fx.decode_weight(m.trellis, m.bits_x2, m.codebook).float()
    return cache[key]
