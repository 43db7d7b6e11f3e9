"""MoE routing and EXL3 expert execution.

GPU path (one call = 6 launches, all CUDA-graph capturable, no host sync):
  moe_topk -> moe_build_assignments (deterministic expert-sorted rows + work
  items) -> exl3_input_rotate (gate/up input rotations, fp16) -> exl3_gemm
  gate/up pass (SwiGLU + down-input rotation fused in the epilogue) ->
  exl3_gemm down pass -> moe_combine (weighted sum over top-k, fixed order).
CPU path: the fp32 oracle of ``oracle.moe``.
"""

from __future__ import annotations

import dataclasses

import torch

from .. import _ext
from ..formats import exl3 as fx
from ..oracle import moe as _ref


@dataclasses.dataclass
class Exl3Experts:
    """Stacked EXL3 expert weights of one MoE layer on one rank.

    gate/up: trellis [E, H/16, I/16, 8*b], suh [E, H], svh [E, I]
    down:    trellis [E, I/16, H/16, 8*b], suh [E, I], svh [E, H]
    ``expert_map`` (int32 [E_global], -1 = not on this rank) for expert parallel.
    """

    gate_trellis: torch.Tensor
    up_trellis: torch.Tensor
    down_trellis: torch.Tensor
    gate_suh: torch.Tensor
    up_suh: torch.Tensor
    down_suh: torch.Tensor
    gate_svh: torch.Tensor
    up_svh: torch.Tensor
    down_svh: torch.Tensor
    bits_x2: int
    codebook: int
    hidden: int
    intermediate: int
    expert_map: torch.Tensor | None = None
    swiglu_limit: float = 0.0

    @property
    def num_local(self) -> int:
        return self.gate_trellis.shape[0]

    @staticmethod
    def from_matrices(gate: list, up: list, down: list, expert_map=None, swiglu_limit=0.0) -> "Exl3Experts":
        g, u, d = fx.stack_experts(gate), fx.stack_experts(up), fx.stack_experts(down)
        return Exl3Experts(g["trellis"], u["trellis"], d["trellis"], g["suh"], u["suh"], d["suh"], g["svh"],
                           u["svh"], d["svh"], gate[0].bits_x2, gate[0].codebook, gate[0].in_features,
                           gate[0].out_features, expert_map, swiglu_limit)

    def select(self, first: int, count: int) -> "Exl3Experts":
        """Experts [first, first + count) (expert-parallel share of a fully drawn layer)."""
        import dataclasses

        sl = slice(first, first + count)
        return dataclasses.replace(self, **{f"{w}_{t}": getattr(self, f"{w}_{t}")[sl].contiguous()
                                            for w in ("gate", "up", "down") for t in ("trellis", "suh", "svh")})

    def matrices(self, which: str, e: int) -> fx.Exl3Matrix:
        t = getattr(self, f"{which}_trellis")[e]
        suh, svh = getattr(self, f"{which}_suh")[e], getattr(self, f"{which}_svh")[e]
        fin, fout = (self.intermediate, self.hidden) if which == "down" else (self.hidden, self.intermediate)
        return fx.Exl3Matrix(t, suh, svh, self.bits_x2, self.codebook, fin, fout)

    def to(self, device) -> "Exl3Experts":
        kw = {f.name: (getattr(self, f.name).to(device) if isinstance(getattr(self, f.name), torch.Tensor) else
                       getattr(self, f.name)) for f in dataclasses.fields(self)}
        return Exl3Experts(**kw)


def topk(logits: torch.Tensor, k: int, mode: int = 0, bias: torch.Tensor | None = None, scale: float = 1.0,
         renorm: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    if not logits.is_cuda:
        return _ref.topk(logits, k, mode, bias, scale, renorm)
    T = logits.shape[0]
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    lf = logits.float().contiguous()
    _ext.ops().moe_topk(lf, k, mode, None if bias is None else bias.float().contiguous(), scale, renorm, ids, w)
    return ids, w


def pick_tile_rows(T: int, k: int, E_local: int) -> int:
    from .. import envs

    forced = envs.get("VLLM_B200_EXL3_TILE_ROWS")
    if forced:
        if forced not in (16, 32, 64, 128):
            raise ValueError(f"VLLM_B200_EXL3_TILE_ROWS={forced}: 16, 32, 64 or 128")
        return forced
    from ..tuning_table import lookup

    avg = max(1, T * k // max(1, E_local))
    for max_avg, tile in lookup("exl3_moe", "tile_rows_by_avg_rows", {}, ((8, 16), (16, 32), (32, 64))):
        if avg <= max_avg:
            return tile
    return 128


def exl3_moe(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, ex: Exl3Experts,
             add: torch.Tensor | None = None, out_f32: bool = False, reduce: bool = False) -> torch.Tensor:
    """Routed EXL3 experts: out[t] = sum_j w[t,j] * expert_{ids[t,j]}(x[t]) (+ add[t]); with `reduce`,
    summed over the tensor-parallel group (bf16; the combine fused with the all-reduce)."""
    T, H = x.shape
    k = ids.shape[1]
    if not x.is_cuda:
        cache = getattr(ex, "_dense_cache", None)
        if cache is None:
            cache = {}
            object.__setattr__(ex, "_dense_cache", cache)
        d = {"gate": [ex.matrices("gate", e) for e in range(ex.num_local)],
             "up": [ex.matrices("up", e) for e in range(ex.num_local)],
             "down": [ex.matrices("down", e) for e in range(ex.num_local)],
             "expert_map": ex.expert_map}
        y = _ref.exl3_experts(x, ids, weights, d, ex.swiglu_limit or None, cache)
        if add is not None:
            y = y + add.float()
        if reduce:
            from ..parallel import comm

            return comm.tp_all_reduce(y.to(x.dtype))
        return y if out_f32 else y.to(x.dtype)
    y, slot_of, sorted_weight = exl3_moe_rows(x, ids, weights, ex)
    return exl3_combine(y, slot_of, sorted_weight, k, add, T, H, reduce, out_f32)


def exl3_combine(y, slot_of, sorted_weight, k: int, add, T: int, H: int, reduce: bool = False,
                 out_f32: bool = False) -> torch.Tensor:
    """The top-k weighted combine of `exl3_moe_rows`' expert outputs (+ add), fused with the all-reduce
    when `reduce`."""
    if reduce:
        from ..parallel import comm

        return comm.combine_all_reduce(y, slot_of, sorted_weight, k, add, T, H)
    out = torch.empty(T, H, dtype=torch.float32 if out_f32 else torch.bfloat16, device=y.device)
    _ext.ops().moe_combine(y, slot_of, sorted_weight, k, add, out)
    return out


def exl3_moe_rows(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, ex: Exl3Experts, build=None):
    """The expert half of `exl3_moe` on CUDA tensors: returns (y [T k, Hp] fp32 expert outputs in
    expert-sorted rows, slot_of [T, k] row of each (token, pick) or -1, sorted_weight [T k]).
    `build` replaces the assignment builder (the sequence-parallel one waits for the dispatch)."""
    T, H = x.shape
    k = ids.shape[1]
    ops = _ext.ops()
    dev = x.device
    E = ex.num_local
    Kh = ex.gate_trellis.shape[1] * 16  # padded hidden
    I = ex.gate_trellis.shape[2] * 16  # padded intermediate
    Hp = ex.down_trellis.shape[2] * 16  # padded hidden out
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
    (build or ops.moe_build_assignments)(ids.contiguous(), weights.float().contiguous(), ex.expert_map, E, tile,
                                         sorted_token, sorted_weight, slot_of, items, num_items, offsets)
    xg = torch.empty(TK, Kh, dtype=torch.float16, device=dev)
    xu = torch.empty(TK, Kh, dtype=torch.float16, device=dev)
    # activation row sums (codebook 2 applies its affine step to the accumulator: a acc + b sum x)
    sg = torch.empty(TK, dtype=torch.float32, device=dev)
    su = torch.empty(TK, dtype=torch.float32, device=dev)
    ops.exl3_input_rotate(x, H, sorted_token, offsets, E, ex.gate_suh, ex.up_suh, xg, xu, TK, sg, su)
    h = torch.empty(TK, I, dtype=torch.float16, device=dev)
    hsum = torch.empty(TK, I // 128, dtype=torch.float32, device=dev)
    st = _ext.status_word(dev)
    ops.exl3_gemm(2, ex.gate_trellis, ex.up_trellis, ex.gate_svh, ex.up_svh, ex.down_suh, ex.bits_x2, ex.codebook,
                  xg, xu, tile, items, num_items, max_items * (I // 128), h, 0, float(ex.swiglu_limit or 0.0), st,
                  sg, su, 1, hsum)
    y = torch.empty(TK, Hp, dtype=torch.float32, device=dev)
    ops.exl3_gemm(1, ex.down_trellis, None, ex.down_svh, None, None, ex.bits_x2, ex.codebook, h, None, tile, items,
                  num_items, max_items * (Hp // 128), y, 1, 0.0, st, hsum, None, I // 128, None)
    return y, slot_of, sorted_weight


_DENSE_ITEMS: dict = {}


def dense_items(T: int, tile: int, dev) -> tuple[torch.Tensor, torch.Tensor]:
    """Work items {expert 0, row0, rows, 0} [n, 4] int32 and their count [1] covering T rows of a dense
    (one-matrix) GEMM.  Built with device ops so CUDA-graph capture can record them; cached per shape
    outside capture (a tensor made during capture holds its values only after a replay)."""
    key = (T, tile, str(dev))
    hit = _DENSE_ITEMS.get(key)
    if hit is not None:
        return hit
    n = (T + tile - 1) // tile
    r = torch.arange(n, dtype=torch.int32, device=dev) * tile
    z = torch.zeros_like(r)
    items = torch.stack([z, r, (T - r).clamp(max=tile), z], dim=1).contiguous()
    num = torch.full((1,), n, dtype=torch.int32, device=dev)
    if not (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()):
        _DENSE_ITEMS[key] = (items, num)
    return items, num


def exl3_linear(x: torch.Tensor, m: fx.Exl3Matrix, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Dense EXL3 linear (one matrix): the MoE kernels with a single expert."""
    if not x.is_cuda:
        return fx.linear(x, m).to(out_dtype)
    ops = _ext.ops()
    T = x.shape[0]
    dev = x.device
    K, N = m.padded_in, m.padded_out
    tile = 128 if T > 64 else (64 if T > 32 else (32 if T > 16 else 16))
    n_items = (T + tile - 1) // tile
    items, num = dense_items(T, tile, dev)
    xr = torch.empty(max(T, 1), K, dtype=torch.float16, device=dev)
    sx = torch.empty(max(T, 1), dtype=torch.float32, device=dev)
    ops.exl3_input_rotate(x, m.in_features, None, None, 1, m.suh, None, xr, None, T, sx, None)
    y = torch.empty(T, N, dtype=torch.float32 if out_dtype == torch.float32 else torch.bfloat16, device=dev)
    ops.exl3_gemm(1, m.trellis.unsqueeze(0), None, m.svh, None, None, m.bits_x2, m.codebook, xr, None, tile, items,
                  num, n_items * (N // 128), y, 1 if out_dtype == torch.float32 else 2, 0.0, _ext.status_word(dev),
                  sx, None, 1, None)
    return y[:, : m.out_features]
