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


class FusedComm:
    """Symmetric buffer of the compute-fused all-reduce kernels.

    Layout per rank: [GEMM flags: cta x 4 lane quarters x src][combine flags: block x src]
    [GEMM tile slots: cta x 2 parities x src x tile][combine slots: 2 parities x src x message].
    Each kernel keeps per-CTA (per-block) call counters as its flag epochs."""

    def __init__(self, group, cpu_group, device: torch.device, max_ctas: int = 160, tile_cap: int = 64 << 10,
                 combine_bytes: int = 4 << 20, combine_blocks: int = 148, timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_ctas, self.tile_cap = max_ctas, tile_cap
        self.combine_bytes, self.combine_blocks = combine_bytes, combine_blocks
        self.timeout_s = timeout_s
        w = self.world

        def up(n):
            return (n + 4095) // 4096 * 4096

        self.gemm_flag_off = 0
        self.comb_flag_off = up(max_ctas * 4 * w * 4)
        flags_end = self.comb_flag_off + up(combine_blocks * w * 4)
        self.gemm_data_off = flags_end
        self.comb_data_off = self.gemm_data_off + max_ctas * 2 * w * tile_cap
        total = self.comb_data_off + 2 * w * combine_bytes
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.buf[:flags_end].zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.peers = torch.tensor(list(self.hdl.buffer_ptrs), dtype=torch.int64, device=device)
        self.gemm_epochs = torch.zeros(max_ctas, dtype=torch.int32, device=device)
        self.comb_epochs = torch.zeros(combine_blocks, dtype=torch.int32, device=device)
        self._fits: dict = {}
        torch.cuda.synchronize(device)
        dist.barrier(group=cpu_group)

    def gemm_all_reduce(self, x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor | None:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        M, N = x2.shape[0], w.shape[0]
        key = (M, N)
        fits = self._fits.get(key)
        if fits is None:
            fits = self._gemm_fits(M, N, x.device)
            self._fits[key] = fits
        if not fits or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
            return None
        if x2.stride(-1) != 1 or (x2.stride(0) % 8 and M > 1):
            x2 = x2.contiguous()
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
        _ext.ops().gemm_allreduce(x2, w, bias, out, self.peers, self.rank, self.world, self.gemm_flag_off,
                                  self.gemm_data_off, self.tile_cap, self.max_ctas, self.gemm_epochs,
                                  _ext.status_word(x.device), self.timeout_s)
        return out.view(*lead, N)

    def _gemm_fits(self, M: int, N: int, device) -> bool:
        """Same rule as gemm_bf16_allreduce_fits (gemm_bf16.cu): one 128-row output tile per CTA, every
        CTA resident, the tile within a slot."""
        swap = M <= 128
        ma, nb = (N, M) if swap else (M, N)
        bn = (16 if nb <= 16 else 32 if nb <= 32 else 64 if nb <= 64 else 128) if swap else 256
        tiles = -(-ma // 128) * -(-nb // bn)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        return tiles <= sms and tiles <= self.max_ctas and 128 * bn * 2 <= self.tile_cap

    def combine_all_reduce(self, y, slot_of, sorted_weight, k: int, add, T: int, H: int) -> torch.Tensor | None:
        if T * H * 2 > self.combine_bytes or H % 8 or y.stride(0) % 4:
            return None
        out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
        _ext.ops().combine_allreduce(y, slot_of, sorted_weight, k, add, out, self.peers, self.rank, self.world,
                                     self.comb_flag_off, self.comb_data_off, self.combine_bytes, self.comb_epochs,
                                     _ext.status_word(y.device), self.timeout_s)
        return out


def _agree(ok: bool, cpu_group) -> bool:
    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=cpu_group)
    return bool(t.item())


def sp_max_tokens(engine) -> int:
    """Largest step the sequence-parallel buffers take: the decode graphs' batch (times the verify
    width), at least 256 tokens; larger steps (prefill chunks) take the all-reduce layout."""
    c = engine.cfg
    from ..tuning_table import lookup

    per = 1 + max(0, c.scheduler.num_speculative_tokens)
    graphs = max(c.cuda_graph_batch_sizes or [0])
    return max(lookup("sp", "min_max_tokens", {}, 256), min(4096, max(graphs, c.scheduler.max_num_seqs) * per))


def enable_for_engine(engine) -> bool:
    """Switch the engine's TP all-reduces to the symmetric-memory kernel when
    every rank can set it up; returns whether it is active."""
    from .. import envs

    st = pstate.get()
    if st.tp_size == 1 or st.device.type != "cuda":
        return False
    transport = envs.get("VLLM_B200_ALLREDUCE")
    if transport not in ("symm", "nccl"):
        raise ValueError(f"VLLM_B200_ALLREDUCE={transport!r}: 'symm' or 'nccl'")
    envs.log_gate("symmetric-memory collectives", transport == "symm", "VLLM_B200_ALLREDUCE=nccl")
    if transport == "nccl":
        return False
    wait_s = envs.get("VLLM_B200_ALLREDUCE_WAIT_S")
    symm = fused = None
    try:
        from ..tuning_table import lookup

        max_bytes = envs.get("VLLM_B200_ALLREDUCE_MAX_BYTES") or lookup("allreduce", "symm_max_bytes", {}, 16 << 20)
        symm = SymmComm(st.tp_group, st.tp_cpu_group, st.device, max_bytes=max_bytes, timeout_s=wait_s)
        ok = True
    except Exception as e:  # noqa: BLE001 -- any setup failure falls back on every rank
        log.warning("symmetric-memory all-reduce unavailable on rank %d: %s", st.rank, e)
        ok = False
    ok = _agree(ok, st.tp_cpu_group)
    fused_ok = False
    if ok and engine.cfg.parallel.fused_comm and envs.get("VLLM_B200_FUSED_GEMM_AR"):
        try:
            fused = FusedComm(st.tp_group, st.tp_cpu_group, st.device, timeout_s=wait_s)
            fused_ok = True
        except Exception as e:  # noqa: BLE001
            log.warning("fused compute + all-reduce kernels unavailable on rank %d: %s", st.rank, e)
        fused_ok = _agree(fused_ok, st.tp_cpu_group)
    comm.enable_fused(symm if ok else None, fused if fused_ok else None)
    model = engine.runner.model
    p = engine.cfg.parallel
    if (ok and p.fused_comm and st.expert_parallel and p.sequence_parallel
            and envs.get("VLLM_B200_EP_DISPATCH") == "symm" and hasattr(model, "supports_sp") and model.supports_sp()):
        from .sp import FusedSP

        sp = None
        try:
            sp = FusedSP(st.tp_group, st.tp_cpu_group, st.device, model.cfg.hidden_size, model.cfg.moe.top_k,
                         max_tokens=sp_max_tokens(engine), timeout_s=wait_s)
            sp_ok = True
        except Exception as e:  # noqa: BLE001 -- any setup failure falls back on every rank
            log.warning("sequence-parallel kernels unavailable on rank %d: %s", st.rank, e)
            sp_ok = False
        if _agree(sp_ok, st.tp_cpu_group):
            comm.enable_sp(sp)
    if st.rank == 0:
        log.info("TP all-reduce: %s", "symmetric-memory one-shot kernel" if ok else "NCCL")
    return ok
