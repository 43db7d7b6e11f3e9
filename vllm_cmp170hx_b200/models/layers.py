"""Model building blocks over the package's ops (tcgen05 kernels on GPU,
oracles on CPU) and the TP collectives.

Weights are created by a :class:`WeightInit` that either draws the full
logical tensor from a seeded CPU generator and keeps this rank's shard
(`mode="sliced"`: the same model at every TP size, used by tests) or draws
only the local shard on the device (`mode="local"`: fast random init of the
BASELINE-sized models for benchmarks).
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .. import ops
from ..parallel import comm
from ..parallel import state as pstate


class WeightInit:
    def __init__(self, seed: int, device, mode: str = "local", dtype=torch.bfloat16):
        self.seed = seed
        self.device = torch.device(device)
        self.mode = mode
        self.dtype = dtype
        self._n = 0

    def _gen(self, device, sharded: bool = False) -> torch.Generator:
        """Generator of the next draw.  In `local` mode a rank's shard of a split tensor gets its own
        stream (rank salt); replicated tensors get the same stream on every rank."""
        self._n += 1
        g = torch.Generator(device=device)
        st = pstate.get()
        salt = 7919 * (st.tp_rank + 1) if (self.mode != "sliced" and sharded) else 0
        g.manual_seed(self.seed * 1000003 + self._n * 9973 + salt)
        return g

    def normal(self, shape, std: float, shard: tuple[int, int, int] | None = None, dtype=None) -> torch.Tensor:
        """shard = (dim, rank, size): keep this rank's contiguous part along dim."""
        dtype = dtype or self.dtype
        if shard is not None and shard[2] == 1:
            shard = None  # a split over one rank is the whole (replicated) tensor
        if self.mode == "sliced" or self.device.type == "cpu":
            t = torch.randn(*shape, generator=self._gen("cpu")) * std
            if shard is not None:
                d, r, n = shard
                t = t.chunk(n, dim=d)[r]
            return t.to(dtype).contiguous().to(self.device)
        local = list(shape)
        if shard is not None:
            d, _, n = shard
            local[d] //= n
        return (torch.randn(*local, generator=self._gen(self.device, shard is not None), device=self.device)
                * std).to(dtype)

    def ones_plus(self, n: int, scale: float = 0.0, dtype=None) -> torch.Tensor:
        t = torch.ones(n) + scale * torch.randn(n, generator=self._gen("cpu"))
        return t.to(dtype or self.dtype).to(self.device)

    def uniform(self, shape, lo: float, hi: float, dtype=torch.float32) -> torch.Tensor:
        t = torch.rand(*shape, generator=self._gen("cpu")) * (hi - lo) + lo
        return t.to(dtype).to(self.device)


class Linear(nn.Module):
    """y = x W^T; weight [out, in] bf16 (this rank's shard)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias, requires_grad=False)

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def forward(self, x: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        return ops.gemm(x, self.weight, self.bias, out_dtype=out_dtype)

    def forward_reduced(self, x: torch.Tensor) -> torch.Tensor:
        """Row-parallel use: the output summed over the tensor-parallel group."""
        return comm.gemm_all_reduce(x, self.weight, self.bias)


class GroupedLinear(nn.Module):
    """Block-diagonal projection: x [T, G, in] -> [T, G * out], output group g = x[:, g] W_g^T.

    bf16 groups run as one GEMM per group straight off the strided input view and into their
    column slice of the output (no copies); fp8 block-scaled groups (`fmt="fp8_block"`, the
    DeepSeek-V4.1 `wo_a` form) go through the fp8 dequant GEMM per group.  The reference runs a
    block-diagonal layer of any linear method group by group the same way
    (vllm_sm80/layers/grouped_linear.py:35-94)."""

    def __init__(self, weights: torch.Tensor, fmt: str = "bf16"):
        super().__init__()
        G, out_g, _ = weights.shape
        self.groups, self.out_g, self.fmt = G, out_g, fmt
        if fmt == "bf16":
            self.weight = nn.Parameter(weights.contiguous(), requires_grad=False)
        elif fmt == "fp8_block":
            from .marlin_experts import Fp8Proj

            self.parts = nn.ModuleList([Fp8Proj(weights[g]) for g in range(G)])
        else:
            raise ValueError(f"unknown grouped linear format {fmt!r}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 3 or x.shape[1] != self.groups:
            raise ValueError(f"grouped input must be [tokens, {self.groups}, in]")
        if self.fmt != "bf16":
            return torch.cat([p(x[:, g]) for g, p in enumerate(self.parts)], dim=-1)
        T = x.shape[0]
        out = torch.empty(T, self.groups * self.out_g, dtype=torch.bfloat16, device=x.device)
        for g in range(self.groups):
            ops.gemm(x[:, g], self.weight[g], out=out[:, g * self.out_g:(g + 1) * self.out_g])
        return out


class RMSNorm(nn.Module):
    def __init__(self, weight: torch.Tensor, eps: float):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.eps = eps

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return ops.rms_norm(x, self.weight, self.eps)
        ops.fused_add_rms_norm(x, residual, self.weight, self.eps)
        return x


def row_parallel_reduce(y: torch.Tensor) -> torch.Tensor:
    return comm.tp_all_reduce(y)


def default_std(fan_in: int) -> float:
    return 1.0 / math.sqrt(fan_in)
