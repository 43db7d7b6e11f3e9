"""Random-init Marlin int4 experts (and fp8 projections) for the DeepSeek-style models."""

from __future__ import annotations

import torch

from ..formats import fp8 as f8
from ..formats import marlin as fm
from ..ops.dequant import Fp8Linear, MarlinExperts
from ..parallel import state as pstate


def random_marlin_experts(E: int, hid: int, inter_local: int, wi, tp: int, tp_rank: int) -> MarlinExperts:
    """Packed int32 codes are drawn uniformly (every word is a valid code);
    scales ~ 1/(4 sqrt(K)) keep activations unit-scale.  `sliced` init draws
    the full intermediate and keeps this rank's columns (gate/up) / rows (down),
    whole 128-wide groups, as the reference's Marlin TP split does."""
    dev = wi.device
    if wi.mode == "sliced":
        g = torch.Generator().manual_seed(wi.seed * 37 + 11)
        inter = inter_local * tp
        gp, gs = fm.random_experts(E, hid, inter, generator=g)
        up, us = fm.random_experts(E, hid, inter, generator=g)
        dp, ds = fm.random_experts(E, inter, hid, generator=g)
        if tp > 1:
            def cut_cols(p, s):  # gate/up: N split, via dense round trip to keep the packed order exact
                outs_p, outs_s = [], []
                for e in range(E):
                    q = _codes(p[e], hid, inter)[:, tp_rank * inter_local:(tp_rank + 1) * inter_local]
                    sc = _scales(s[e], inter)[:, tp_rank * inter_local:(tp_rank + 1) * inter_local]
                    pp, ss = fm.pack(q, sc)
                    outs_p.append(pp)
                    outs_s.append(ss)
                return torch.stack(outs_p), torch.stack(outs_s)

            def cut_rows(p, s):  # down: K split (whole groups of 128)
                outs_p, outs_s = [], []
                for e in range(E):
                    q = _codes(p[e], inter, hid)[tp_rank * inter_local:(tp_rank + 1) * inter_local]
                    sc = _scales(s[e], hid)[tp_rank * inter_local // 128:(tp_rank + 1) * inter_local // 128]
                    pp, ss = fm.pack(q, sc)
                    outs_p.append(pp)
                    outs_s.append(ss)
                return torch.stack(outs_p), torch.stack(outs_s)

            gp, gs = cut_cols(gp, gs)
            up, us = cut_cols(up, us)
            dp, ds = cut_rows(dp, ds)
        return MarlinExperts(gp.to(dev), gs.to(dev), up.to(dev), us.to(dev), dp.to(dev), ds.to(dev), hid, inter_local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(wi.seed * 13 + 1000 * pstate.get().rank + 7)

    def packed(k, n):
        return torch.randint(-(1 << 31), 1 << 31, (E, k // 16, 2 * n), dtype=torch.int64, device=dev,
                             generator=gen).to(torch.int32)

    def scales(k, n):
        return ((torch.rand(E, k // 128, n, device=dev, generator=gen) * 0.5 + 0.75) * (0.25 / k ** 0.5)).to(
            torch.bfloat16)

    return MarlinExperts(packed(hid, inter_local), scales(hid, inter_local), packed(hid, inter_local),
                         scales(hid, inter_local), packed(inter_local, hid), scales(inter_local, hid), hid, inter_local)


def _codes(packed: torch.Tensor, K: int, N: int) -> torch.Tensor:
    k, n = fm._index_maps(K, N)
    words = packed.reshape(K // 16, N // 64, 32, 4).to(torch.int64) & 0xFFFFFFFF
    q = torch.zeros(K, N, dtype=torch.int64)
    for i in range(8):
        q[k[..., i], n[..., i]] = (words >> (4 * i)) & 15
    return q


def _scales(stored: torch.Tensor, N: int) -> torch.Tensor:
    s = torch.empty_like(stored)
    s[:, fm.scale_perm(N)] = stored
    return s


class Fp8Proj(torch.nn.Module):
    """fp8 block-scaled projection (the DeepSeek checkpoint convention)."""

    def __init__(self, w: torch.Tensor):
        super().__init__()
        q, s = f8.quantize(w.float().cpu())
        self.lin = Fp8Linear(q.to(w.device), s.to(w.device))

    @property
    def out_features(self) -> int:
        return self.lin.weight.shape[0]

    def forward(self, x: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        y = self.lin(x)
        return y if out_dtype == torch.bfloat16 else y.to(out_dtype)

    def forward_reduced(self, x: torch.Tensor) -> torch.Tensor:
        from ..parallel import comm

        return comm.tp_all_reduce(self.lin(x))
