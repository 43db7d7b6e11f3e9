"""Tensor-parallel collectives used by the models.

Two paths, chosen per process (all ranks agree: the choice depends only on
the configuration and the message size):

* the NCCL baseline (``torch.distributed`` on the TP group);
* the product path: this package's own kernels over NVLink peer memory
  (symmetric buffers, ``parallel/symm.py``) -- a one-shot all-reduce for
  decode-sized messages and the fused GEMM + reduce-scatter / all-gather +
  GEMM kernels of the row/column-parallel projections.

The reference's equivalent dispatch is Sm80CudaCommunicator.all_reduce
(vllm_sm80/distributed/communicator.py:545): host-staged -> flags-in-data P2P
-> NCCL.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import state as _state

_FUSED = {"enabled": False, "symm": None, "fused": None, "sp": None}


def enable_fused(symm, fused=None) -> None:
    """Route TP all-reduces through the symmetric-memory kernels of `symm`, and the row-parallel
    projections / MoE combines through the compute-fused kernels of `fused`."""
    _FUSED["enabled"] = symm is not None
    _FUSED["symm"] = symm
    _FUSED["fused"] = fused


def fused_enabled() -> bool:
    return _FUSED["enabled"]


def enable_sp(sp) -> None:
    """Run expert-parallel steps that fit `sp` (a parallel.sp transport) in the sequence-parallel layout."""
    _FUSED["sp"] = sp


def sp_for(T: int, model):
    """The sequence-parallel transport for a step of T tokens of `model`, or None (all-reduce layout)."""
    sp = _FUSED["sp"]
    if sp is None or not sp.fits(T):
        return None
    ok = getattr(model, "_sp_ok", None)
    if ok is None:
        ok = model.supports_sp()
        model._sp_ok = ok
    return sp if ok else None


def tp_all_reduce(x: torch.Tensor) -> torch.Tensor:
    from . import sp as _sp

    st = _state.get()
    spa = _sp.active()
    if spa is not None:  # a row-parallel output inside the sequence-parallel layout
        spa.rs_tensor(x.reshape(-1, x.shape[-1]))
        return None
    if st.tp_size == 1 or st.emulated:
        return x
    symm = _FUSED["symm"]
    if _FUSED["enabled"] and symm is not None and symm.can_all_reduce(x):
        return symm.all_reduce(x)
    dist.all_reduce(x, group=st.tp_group)
    return x


def tp_all_gather(x: torch.Tensor, dim: int = 0) -> torch.Tensor:
    st = _state.get()
    if st.tp_size == 1:
        return x
    if st.emulated:
        return torch.cat([x] * st.tp_size, dim=dim)
    parts = [torch.empty_like(x) for _ in range(st.tp_size)]
    dist.all_gather(parts, x.contiguous(), group=st.tp_group)
    return torch.cat(parts, dim=dim)


def tp_all_gather_into(out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """out [tp * n, ...] <- concatenation of every rank's x [n, ...] (rank order)."""
    st = _state.get()
    if st.tp_size == 1 or st.emulated:
        out.copy_(x.repeat(out.shape[0] // x.shape[0], *([1] * (x.dim() - 1))))
        return out
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def tp_reduce_scatter(x: torch.Tensor) -> torch.Tensor:
    """x [tp * n, ...] summed over ranks; returns this rank's [n, ...] slice."""
    st = _state.get()
    if st.tp_size == 1:
        return x
    if st.emulated:
        return x[: x.shape[0] // st.tp_size]
    out = torch.empty(x.shape[0] // st.tp_size, *x.shape[1:], dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def gemm_all_reduce(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Row-parallel projection: sum over the TP group of x @ w^T (+ bias once).  Product path: one
    kernel computes the GEMM tile, pushes it to every rank and sums the pushed tiles (gemm_bf16.cu);
    baseline: GEMM, then the all-reduce."""
    from .. import ops
    from . import sp as _sp

    st = _state.get()
    spa = _sp.active()
    if spa is not None:  # sequence-parallel layout: reduce-scatter to the token owners instead
        if bias is not None:
            raise ValueError("sequence-parallel row-parallel projections take no bias")
        spa.gemm_rs(x.reshape(-1, x.shape[-1]), w)
        return None
    if st.tp_size == 1:
        return ops.gemm(x, w, bias)
    fc = _FUSED["fused"]
    if fc is not None and x.is_cuda:
        y = fc.gemm_all_reduce(x, w, bias)
        if y is not None:
            return y
    y = tp_all_reduce(ops.gemm(x, w))
    return y if bias is None else y + bias


def combine_all_reduce(y: torch.Tensor, slot_of: torch.Tensor, sorted_weight: torch.Tensor, k: int,
                       add: torch.Tensor | None, T: int, H: int) -> torch.Tensor:
    """MoE output: out[t] = sum_j w * y[slot] (+ add[t]), summed over the TP group (bf16 [T, H]).
    Product path: the combine and the all-reduce in one kernel (fused_comm.cu)."""
    from .. import _ext

    st = _state.get()
    fc = _FUSED["fused"]
    if st.tp_size > 1 and fc is not None and y.is_cuda:
        out = fc.combine_all_reduce(y, slot_of, sorted_weight, k, add, T, H)
        if out is not None:
            return out
    out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
    _ext.ops().moe_combine(y, slot_of, sorted_weight, k, add, out)
    return tp_all_reduce(out)
