"""Marlin int4 (group 128) experts and fp8 block-scaled linears on the
dequantizing tcgen05 GEMM (csrc/dequant_gemm.cu); CPU tensors take the
format oracles of ``formats/``."""

from __future__ import annotations

import dataclasses

import torch

from .. import _ext
from ..formats import fp8 as f8
from ..formats import marlin as fm
from .moe import dense_items, pick_tile_rows


@dataclasses.dataclass
class MarlinExperts:
    """Per layer and rank: packed int32 [E, K/16, 2N] and stored-order bf16 scales [E, K/128, N]
    for gate/up (K = hidden, N = intermediate) and down (K = intermediate, N = hidden)."""

    gate: torch.Tensor
    gate_s: torch.Tensor
    up: torch.Tensor
    up_s: torch.Tensor
    down: torch.Tensor
    down_s: torch.Tensor
    hidden: int
    intermediate: int
    expert_map: torch.Tensor | None = None
    swiglu_limit: float = 0.0

    @property
    def num_local(self) -> int:
        return self.gate.shape[0]

    def select(self, first: int, count: int) -> "MarlinExperts":
        """Experts [first, first + count) (expert-parallel share of a fully drawn layer)."""
        sl = slice(first, first + count)
        return dataclasses.replace(self, **{n: getattr(self, n)[sl].contiguous()
                                            for n in ("gate", "gate_s", "up", "up_s", "down", "down_s")})

    def dense(self, which: str, e: int) -> torch.Tensor:
        """Dequantized [K, N] weight of one expert (oracle path)."""
        return fm.unpack(getattr(self, which)[e].cpu(), getattr(self, which + "_s")[e].cpu())


def _moe_cpu(x, ids, w, ex: MarlinExperts) -> torch.Tensor:
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32)
    cache = getattr(ex, "_dense", None)
    if cache is None:
        cache = {}
        object.__setattr__(ex, "_dense", cache)
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e < 0:  # an expert of another rank (masked id)
                continue
            if ex.expert_map is not None:
                e = int(ex.expert_map[e])
                if e < 0:
                    continue
            if e not in cache:
                cache[e] = tuple(ex.dense(n, e).float() for n in ("gate", "up", "down"))
            G, U, D = cache[e]
            xf = x[t].float()
            g, u = xf @ G, xf @ U
            if ex.swiglu_limit:
                g = g.clamp(max=ex.swiglu_limit)
                u = u.clamp(-ex.swiglu_limit, ex.swiglu_limit)
            h = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
            out[t] += float(w[t, j]) * (h @ D)
    return out


def marlin_moe(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, ex: MarlinExperts,
               add: torch.Tensor | None = None, out_f32: bool = False, reduce: bool = False) -> torch.Tensor:
    T, H = x.shape
    k = ids.shape[1]
    if not x.is_cuda:
        y = _moe_cpu(x, ids, weights, ex)
        if add is not None:
            y = y + add.float()
        if reduce:
            from ..parallel import comm

            return comm.tp_all_reduce(y.to(x.dtype))
        return y if out_f32 else y.to(x.dtype)
    ops = _ext.ops()
    dev = x.device
    E = ex.num_local
    I = ex.gate.shape[2] // 2
    TK = T * k
    tile = pick_tile_rows(T, k, E)
    max_items = E + (TK + tile - 1) // tile
    i32 = dict(dtype=torch.int32, device=dev)
    sorted_token = torch.empty(TK, **i32)
    sorted_weight = torch.empty(TK, dtype=torch.float32, device=dev)
    slot_of = torch.empty(TK, **i32)
    items = torch.empty(max_items, 4, **i32)
    num_items = torch.empty(1, **i32)
    offsets = torch.empty(E + 1, **i32)
    ops.moe_build_assignments(ids.contiguous(), weights.float().contiguous(), ex.expert_map, E, tile, sorted_token,
                              sorted_weight, slot_of, items, num_items, offsets)
    xs = torch.empty(TK, H, dtype=torch.bfloat16, device=dev)
    ops.gather_rows(x, sorted_token, xs, TK)
    st = _ext.status_word(dev)
    h = torch.empty(TK, I, dtype=torch.bfloat16, device=dev)
    ops.dequant_gemm(0, 2, ex.gate, ex.up, ex.gate_s, ex.up_s, xs, xs, tile, items, num_items, max_items * (I // 128),
                     h, 0, float(ex.swiglu_limit or 0.0), st)
    y = torch.empty(TK, H, dtype=torch.float32, device=dev)
    ops.dequant_gemm(0, 1, ex.down, None, ex.down_s, None, h, None, tile, items, num_items, max_items * (H // 128), y,
                     1, 0.0, st)
    if reduce:
        from ..parallel import comm

        return comm.combine_all_reduce(y, slot_of, sorted_weight, k, add, T, H)
    out = torch.empty(T, H, dtype=torch.float32 if out_f32 else torch.bfloat16, device=dev)
    ops.moe_combine(y, slot_of, sorted_weight, k, add, out)
    return out


@dataclasses.dataclass
class Fp8Linear:
    """y = x W^T with W [N, K] e4m3 and fp32 scales per 128 x 128 block."""

    weight: torch.Tensor  # [N, K] float8_e4m3fn
    scale: torch.Tensor  # [N/128, K/128] fp32

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return fp8_linear(x, self)


def fp8_linear(x: torch.Tensor, lin: Fp8Linear) -> torch.Tensor:
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    N = lin.weight.shape[0]
    if not x.is_cuda:
        W = f8.dequantize(lin.weight.float().to(torch.float8_e4m3fn) if lin.weight.dtype != torch.float8_e4m3fn
                          else lin.weight, lin.scale)
        return (x2.float() @ W.t()).to(torch.bfloat16).view(*lead, N)
    ops = _ext.ops()
    dev = x.device
    tile = 128 if T > 64 else (64 if T > 32 else (32 if T > 16 else 16))
    n_items = (T + tile - 1) // tile
    items, num = dense_items(T, tile, dev)
    xh = torch.empty(T, K, dtype=torch.float16, device=dev)
    ops.gather_rows(x2 if x2.stride(-1) == 1 else x2.contiguous(), None, xh, T)
    out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
    ops.dequant_gemm(1, 1, lin.weight.view(torch.uint8).unsqueeze(0), None, lin.scale.unsqueeze(0), None, xh, None,
                     tile, items, num, n_items * (N // 128), out, 2, 0.0, _ext.status_word(dev))
    return out.view(*lead, N)
