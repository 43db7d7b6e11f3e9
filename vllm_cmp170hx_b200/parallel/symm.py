"""Symmetric-memory collectives of the tensor-parallel group (product path).

PyTorch's symmetric-memory allocator provides the plumbing: one buffer per
rank, mapped into every peer's address space over NVLink, and the exchange
of the peers' base addresses.  The collective itself is this package's CUDA
kernel (``csrc/comm.cu``): a one-shot all-reduce by peer loads with
per-block epoch flags, bounded waits and fp32 rank-order accumulation.

Buffer layout (per rank): [flags: 64 KiB][data half 0][data half 1].
Every setup step ends in an agreement over the CPU group, so either all
ranks use the kernel or none does (the reference's rule for its custom
transports, vllm_sm80/distributed/host_shm_all_reduce.py:64-70).
"""

from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from .. import _ext
from . import comm
from . import state as pstate

log = logging.getLogger(__name__)

FLAG_BYTES = 64 * 1024


class SymmComm:
    def __init__(self, group, cpu_group, device: torch.device, max_bytes: int = 16 << 20, blocks: int = 48,
                 timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_bytes = max_bytes
        self.blocks = blocks
        self.timeout_s = timeout_s
        self.device = device
        total = FLAG_BYTES + 2 * max_bytes
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.buf[:FLAG_BYTES].zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.peers = torch.tensor(list(self.hdl.buffer_ptrs), dtype=torch.int64, device=device)
        self.epochs = torch.zeros(blocks, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=cpu_group)

    def can_all_reduce(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.numel() % 8 == 0
                and x.numel() * 2 <= self.max_bytes)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        _ext.ops().symm_all_reduce(x, out, self.peers, self.rank, self.world, FLAG_BYTES, self.max_bytes,
                                   self.epochs, _ext.status_word(x.device), self.timeout_s)
        return out


def _agree(ok: bool, cpu_group) -> bool:
    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=cpu_group)
    return bool(t.item())


def enable_for_engine(engine) -> bool:
    """Switch the engine's TP all-reduces to the symmetric-memory kernel when
    every rank can set it up; returns whether it is active."""
    st = pstate.get()
    if st.tp_size == 1 or st.device.type != "cuda":
        return False
    symm = None
    try:
        symm = SymmComm(st.tp_group, st.tp_cpu_group, st.device)
        ok = True
    except Exception as e:  # noqa: BLE001 -- any setup failure falls back on every rank
        log.warning("symmetric-memory all-reduce unavailable on rank %d: %s", st.rank, e)
        ok = False
    ok = _agree(ok, st.tp_cpu_group)
    comm.enable_fused(symm if ok else None)
    if st.rank == 0:
        log.info("TP all-reduce: %s", "symmetric-memory one-shot kernel" if ok else "NCCL")
    return ok
