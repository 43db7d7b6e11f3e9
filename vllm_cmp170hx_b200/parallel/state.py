"""Process-group state: one process per GPU, torch.distributed with NCCL for
device collectives and a gloo group for host-side agreement (the reference's
GroupCoordinator split, vllm_sm80/distributed/communicator.py:1-54).

Layout: world = pp * tp; rank r is (pp_rank = r // tp, tp_rank = r % tp).
Environment: RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT
(torchrun).  Every group gets a short timeout so a rank that never arrives
turns into an error on the others instead of a hang.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    tp_size: int = 1
    tp_rank: int = 0
    pp_size: int = 1
    pp_rank: int = 0
    tp_group: object = None  # device group (NCCL) or None
    tp_cpu_group: object = None  # gloo
    pp_group: object = None
    pp_cpu_group: object = None  # gloo group of the same ranks as pp_group
    world_cpu_group: object = None
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))
    backend: str = "none"
    # routed experts split whole across the TP group (expert parallel) instead of by intermediate columns
    expert_parallel: bool = False
    # one process standing in for rank 0 of a tp_size group (per-rank kernel profiling): every
    # collective returns local data, so the numbers are wrong but each kernel gets its per-rank shape
    emulated: bool = False

    @property
    def is_first_pp(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_pp(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    def pp_peer(self, stage: int) -> int:
        """Global rank of pipeline stage `stage` in this rank's TP column."""
        return stage * self.tp_size + self.tp_rank

    def tp_ranks(self) -> list[int]:
        base = self.pp_rank * self.tp_size
        return list(range(base, base + self.tp_size))


_STATE = ParallelState()


def get() -> ParallelState:
    return _STATE


def set_state(s: ParallelState) -> None:
    global _STATE
    _STATE = s


def init(tp_size: int = 1, pp_size: int = 1, backend: str | None = None, timeout_s: float = 120.0,
         device: str | None = None) -> ParallelState:
    """Initialise (or reuse) the default process group and the TP/PP groups."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if tp_size * pp_size != world:
        raise ValueError(f"tp({tp_size}) * pp({pp_size}) != world size ({world})")
    use_cuda = (device or ("cuda" if torch.cuda.is_available() else "cpu")).startswith("cuda")
    if use_cuda:
        torch.cuda.set_device(local_rank)
        dev = torch.device("cuda", local_rank)
    else:
        dev = torch.device("cpu")
    st = ParallelState(rank=rank, world_size=world, local_rank=local_rank, tp_size=tp_size, tp_rank=rank % tp_size,
                       pp_size=pp_size, pp_rank=rank // tp_size, device=dev)
    if world == 1:
        set_state(st)
        return st
    be = backend or ("nccl" if use_cuda else "gloo")
    to = datetime.timedelta(seconds=timeout_s)
    if not dist.is_initialized():
        kw = dict(backend=be, rank=rank, world_size=world, timeout=to)
        if be == "nccl":
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    st.backend = be
    st.world_cpu_group = dist.new_group(backend="gloo", timeout=to)
    for p in range(pp_size):
        ranks = list(range(p * tp_size, (p + 1) * tp_size))
        g = dist.new_group(ranks, backend=be, timeout=to)
        gc = dist.new_group(ranks, backend="gloo", timeout=to)
        if p == st.pp_rank:
            st.tp_group, st.tp_cpu_group = g, gc
    for t in range(tp_size):
        ranks = [p * tp_size + t for p in range(pp_size)]
        g = dist.new_group(ranks, backend=be, timeout=to)
        gc = dist.new_group(ranks, backend="gloo", timeout=to)
        if t == st.tp_rank:
            st.pp_group, st.pp_cpu_group = g, gc
    set_state(st)
    return st


def emulate(tp_size: int, device: str = "cuda") -> ParallelState:
    """Single-process stand-in for rank 0 of a `tp_size` TP group (no process group).  Only for
    measuring per-rank kernel costs of a layout whose GPUs are not at hand."""
    dev = torch.device(device, 0) if device.startswith("cuda") else torch.device("cpu")
    st = ParallelState(tp_size=tp_size, tp_rank=0, device=dev, backend="emulated", emulated=True)
    set_state(st)
    return st


def destroy() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
    set_state(ParallelState())
