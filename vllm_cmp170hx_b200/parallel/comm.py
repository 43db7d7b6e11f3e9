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

_FUSED = {"enabled": False, "symm": None}


def enable_fused(symm) -> None:
    """Route TP all-reduces through the symmetric-memory kernels of `symm`."""
    _FUSED["enabled"] = symm is not None
    _FUSED["symm"] = symm


def fused_enabled() -> bool:
    return _FUSED["enabled"]


def tp_all_reduce(x: torch.Tensor) -> torch.Tensor:
    st = _state.get()
    if st.tp_size == 1:
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
    parts = [torch.empty_like(x) for _ in range(st.tp_size)]
    dist.all_gather(parts, x.contiguous(), group=st.tp_group)
    return torch.cat(parts, dim=dim)


def tp_all_gather_into(out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """out [tp * n, ...] <- concatenation of every rank's x [n, ...] (rank order)."""
    st = _state.get()
    if st.tp_size == 1:
        out.copy_(x)
        return out
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def tp_reduce_scatter(x: torch.Tensor) -> torch.Tensor:
    """x [tp * n, ...] summed over ranks; returns this rank's [n, ...] slice."""
    st = _state.get()
    if st.tp_size == 1:
        return x
    out = torch.empty(x.shape[0] // st.tp_size, *x.shape[1:], dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=st.tp_group)
    return out
