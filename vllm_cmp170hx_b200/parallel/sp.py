"""Sequence-parallel layout of expert-parallel steps, and its two transports.

With expert parallelism (whole experts per rank) and tensor-parallel attention, a step of T tokens
keeps the residual stream sharded by tokens: rank r owns tokens [r Tr, (r + 1) Tr), Tr = T / world.
Per layer the data moves four times:

* all-gather: the normalised rows of every rank, so the column-parallel attention (or dense MLP)
  projection sees all T tokens;
* reduce-scatter: the row-parallel output projection's partial rows, summed at each token's owner;
* dispatch: each token's MoE input row, sent once to every rank that holds one of its top-k experts,
  with its (expert, weight) list;
* combine: each rank's weighted expert sum of a received row, sent back to the token's owner and
  summed there.

Router, shared expert, norms and residual adds then run on Tr tokens per rank instead of T.

Two transports implement the same calls (the model code does not change between them):

* `FusedSP` -- this package's kernels over NVLink peer memory (csrc/sp_comm.cu, the reduce-scatter
  and all-gather modes of the GEMM, the waiting assignment builder): every transfer is a plain peer
  store issued by the kernel that produced the data, and the consumer waits on per-source flags;
* `TorchSP` -- torch.distributed collectives (NCCL on GPUs, gloo in CPU tests): all-gather,
  reduce-scatter, and the reference's expert-parallel scheme (dispatch by all-gather, combine by
  reduce-scatter, vllm_sm80/kernels/exl3/quant.py:1913-1934).  It is the baseline the fused path is
  measured against and the path the CPU tests exercise.
"""

from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from .. import _ext, ops
from . import state as pstate

log = logging.getLogger(__name__)

CH_AG, CH_RS, CH_DISPATCH, CH_COMBINE = 0, 1, 2, 3
FLAG_BYTES = 4096


def _bf16_add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (a.float() + b.float()).to(torch.bfloat16)


class _Base:
    """What both transports share: sizes of the current step and the torch-side math of the norms."""

    fused = False

    def __init__(self, world: int, rank: int, hidden: int, top_k: int, max_tokens: int):
        self.world, self.rank, self.H, self.k = world, rank, hidden, top_k
        self.max_tokens = max_tokens
        self.T = self.Tr = 0

    def fits(self, T: int) -> bool:
        return T > 0 and T % self.world == 0 and T <= self.max_tokens

    def begin(self, T: int) -> int:
        self.T, self.Tr = T, T // self.world
        return self.Tr

    def local_slice(self, t: torch.Tensor) -> torch.Tensor:
        return t[self.rank * self.Tr:(self.rank + 1) * self.Tr]

    def apply(self, pending: tuple, residual: torch.Tensor, w: torch.Tensor, eps: float, ag: bool = False,
              out: torch.Tensor | None = None):
        """The residual update a layer left pending (see DecoderLayer.forward_sp), then the norm."""
        src, arg = pending
        return self.norm(src, residual, w, eps, x=arg if src in ("local", "add") else None,
                         add=arg if src == "comb" else None, ag=ag, out=out)


class TorchSP(_Base):
    """The layout over torch.distributed collectives of the tensor-parallel group."""

    def __init__(self, group, hidden: int, top_k: int, max_tokens: int = 1 << 16):
        st = pstate.get()
        super().__init__(st.tp_size, st.tp_rank, hidden, top_k, max_tokens)
        self.group = group
        self._gathered = None
        self._rs = None
        self._recv = None
        self._dmask = None

    def _all_gather(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty(self.world * x.shape[0], *x.shape[1:], dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def _reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type == "cpu":  # gloo has no reduce-scatter: all-reduce (same sum) and keep this rank's rows
            y = x.float().contiguous()
            dist.all_reduce(y, group=self.group)
            return self.local_slice(y).to(x.dtype)
        out = torch.empty(x.shape[0] // self.world, *x.shape[1:], dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return out

    # ---------------------------------------------------------------- residual + norm (+ all-gather)
    def norm(self, src: str, residual: torch.Tensor, w: torch.Tensor, eps: float, x: torch.Tensor | None = None,
             add: torch.Tensor | None = None, ag: bool = False, out: torch.Tensor | None = None):
        if src == "local":
            residual.copy_(x)
        elif src == "add":
            residual.copy_(_bf16_add(residual, x))
        else:
            y = self._rs if src == "rs" else self._comb
            if src == "comb" and add is not None:
                y = _bf16_add(y, add)
            residual.copy_(_bf16_add(residual, y))
        h = ops.rms_norm(residual, w, eps)
        if out is not None:
            out.copy_(h)
        if ag:
            self._gathered = self._all_gather(h)
        return h

    def gathered(self, wait: bool = False) -> torch.Tensor:
        return self._gathered

    # ---------------------------------------------------------------- row-parallel output
    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor) -> None:
        self._rs = self._reduce_scatter(ops.gemm(x, w))

    def rs_tensor(self, y: torch.Tensor) -> None:
        self._rs = self._reduce_scatter(y)

    # ---------------------------------------------------------------- MoE dispatch / combine
    def route_dispatch(self, logits, h, k, mode, bias, scale, renorm, e_per_rank):
        from ..ops import moe as moe_ops

        ids, wts = moe_ops.topk(logits, k, mode, bias, scale, renorm)
        x_all = self._all_gather(h)
        ids_all = self._all_gather(ids)
        w_all = self._all_gather(wts)
        mine = torch.div(ids_all, e_per_rank, rounding_mode="floor") == self.rank
        self._recv = (x_all, torch.where(mine, ids_all, -1).to(torch.int32).contiguous(), w_all.contiguous())
        return ids, wts

    def dispatch_recv(self):
        return self._recv

    def combine_partial(self, partial: torch.Tensor) -> None:
        """partial [T, H]: this rank's weighted expert sum of every received row (zero without an expert
        here), summed over the ranks at each token's owner."""
        self._comb = self._reduce_scatter(partial.to(torch.bfloat16))


class FusedSP(_Base):
    """The layout over this package's kernels and a symmetric buffer per rank (NVLink peer stores)."""

    fused = True

    def __init__(self, group, cpu_group, device: torch.device, hidden: int, top_k: int, max_tokens: int = 1024,
                 timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem

        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        max_tokens -= max_tokens % world
        super().__init__(world, rank, hidden, top_k, max_tokens)
        self.timeout_s = timeout_s
        self.device = device
        T, H, k = max_tokens, hidden, top_k

        def up(n):
            return (n + 255) // 256 * 256

        off = FLAG_BYTES
        self.ag_off = off
        off += up(T * H * 2)
        self.rs_off = off
        off += up(T * H * 2)
        self.rows_off = off
        off += up(T * H * 2)
        self.ids_off = off
        off += up(T * k * 4)
        self.w_off = off
        off += up(T * k * 4)
        self.comb_off = off
        off += up(T * H * 2)
        self.buf = symm_mem.empty(off, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.peers = torch.tensor(list(self.hdl.buffer_ptrs), dtype=torch.int64, device=device)
        self.state = torch.zeros(16, dtype=torch.int32, device=device)
        self.dmask = torch.zeros(T // world, dtype=torch.int32, device=device)
        self.status = _ext.status_word(device)
        self._pending = None  # data_ptr of the all-gather area while no kernel waited on it yet
        torch.cuda.synchronize(device)

    def _area(self, off: int, rows: int, cols: int, dtype) -> torch.Tensor:
        nbytes = rows * cols * torch.empty((), dtype=dtype).element_size()
        return self.buf[off:off + nbytes].view(dtype).view(rows, cols)

    def _sync(self):
        return (self.peers, self.rank, self.state, self.status, self.timeout_s)

    # ---------------------------------------------------------------- residual + norm (+ all-gather)
    def norm(self, src: str, residual: torch.Tensor, w: torch.Tensor, eps: float, x: torch.Tensor | None = None,
             add: torch.Tensor | None = None, ag: bool = False, out: torch.Tensor | None = None):
        code = {"local": 0, "rs": 1, "comb": 2, "add": 3}[src]
        _ext.ops().sp_residual_norm(*self._sync(), code, x, add, self.dmask if code == 2 else None, self.rs_off,
                                    self.comb_off, self.ag_off, residual, w, float(eps), out, ag)
        if ag:
            self._pending = self.buf.data_ptr() + self.ag_off
        return out

    def gathered(self, wait: bool = False) -> torch.Tensor:
        """The all-gather area [T, H].  Its first reader must wait for the flags: a GEMM through `ops.gemm`
        does so in its producer (all-gather mode); `wait=True` launches a wait for other readers."""
        t = self._area(self.ag_off, self.T, self.H, torch.bfloat16)
        if wait and self._pending is not None:
            _ext.ops().sp_wait(*self._sync(), CH_AG)
            self._pending = None
        return t

    def take_pending(self, x: torch.Tensor) -> bool:
        """Whether `x` is the all-gather area with no waiting reader yet (then the caller waits)."""
        if self._pending is not None and x.data_ptr() == self._pending:
            self._pending = None
            return True
        return False

    def gemm_ag(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        _ext.ops().gemm_sp(x, w, out, self.status, 0, self.peers, self.rank, self.state, self.timeout_s, 2, 0, 0)

    # ---------------------------------------------------------------- row-parallel output
    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor) -> None:
        _ext.ops().gemm_sp(x, w, None, self.status, 0, self.peers, self.rank, self.state, self.timeout_s, 1,
                           self.rs_off, self.Tr)

    # ---------------------------------------------------------------- MoE dispatch / combine
    def route_dispatch(self, logits, h, k, mode, bias, scale, renorm, e_per_rank):
        _ext.ops().sp_route_dispatch(*self._sync(), logits.float().contiguous(), h, k, mode,
                                     None if bias is None else bias.float().contiguous(), float(scale), bool(renorm),
                                     e_per_rank, self.rows_off, self.ids_off, self.w_off, self.dmask, None, None)
        return None, None

    def dispatch_recv(self):
        return (self._area(self.rows_off, self.T, self.H, torch.bfloat16),
                self._area(self.ids_off, self.T, self.k, torch.int32),
                self._area(self.w_off, self.T, self.k, torch.float32))

    def build_assignments(self, ids, weights, expert_map, E_local, tile, sorted_token, sorted_weight, slot_of, items,
                          num_items, offsets) -> None:
        _ext.ops().moe_build_assignments_sp(ids, weights, expert_map, E_local, tile, sorted_token, sorted_weight,
                                            slot_of, items, num_items, offsets, *self._sync())

    def combine_push(self, y: torch.Tensor, slot_of: torch.Tensor, sorted_weight: torch.Tensor, k: int) -> None:
        _ext.ops().sp_combine_push(*self._sync(), y, slot_of, sorted_weight, k, self.comb_off, self.Tr, self.H,
                                   CH_COMBINE)

    def rs_tensor(self, y: torch.Tensor) -> None:
        """A row-parallel output computed by another kernel ([T, H]): each token row to its owner."""
        slot = torch.arange(self.T, device=y.device, dtype=torch.int32)
        _ext.ops().sp_combine_push(*self._sync(), y.float().contiguous(), slot, torch.ones(self.T, device=y.device),
                                   1, self.rs_off, self.Tr, self.H, CH_RS)

    def combine_partial(self, partial: torch.Tensor) -> None:
        """partial [T, H] rows of the received tokens (any expert format): pushed as one-slot combines."""
        ids = self.dispatch_recv()[1]
        has = (ids >= 0).any(1)
        slot = torch.where(has, torch.arange(self.T, device=ids.device, dtype=torch.int32), -1).to(torch.int32)
        self.combine_push(partial.float().contiguous(), slot.contiguous(), torch.ones(self.T, device=ids.device), 1)


_ACTIVE: dict = {"sp": None}


def active():
    return _ACTIVE["sp"]


class scope:
    """Inside: the row-parallel projections reduce-scatter through `sp` (see comm.gemm_all_reduce)."""

    def __init__(self, sp):
        self.sp = sp

    def __enter__(self):
        _ACTIVE["sp"] = self.sp
        return self.sp

    def __exit__(self, *exc):
        _ACTIVE["sp"] = None
        return False
