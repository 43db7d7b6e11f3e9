"""Per-layer-embedding (PLE) lookups from an EXL3-coded table file, decoded on the GPU.

``PleTable(path, prefix, owner_lo, owner_hi)`` serves ``lookup(ids [T, heads]) -> (rows bf16
[T, heads*dim], failed [T])`` for the n-gram ids a model computes per token:

1. ids outside ``[owner_lo, owner_hi)`` (another tensor-parallel rank's rows) or outside every
   head's vocabulary are not read; the others go through the native ``RowCache``
   (``csrc/row_store.cpp``: set-associative LRU host cache, misses ``pread`` on a thread pool
   with retries, the trellis found at its byte offset in the safetensors file) into pinned memory;
2. one asynchronous host->device copy of the packed rows and of the failed-row flags;
3. ``ple_decode`` (``csrc/rows.cu``) decodes the rows (zero rows for ids this rank does not own,
   NaN rows for reads that failed);
4. with a process group, an all-reduce sums the ranks' rows (each id has one owner; NaN survives
   the sum, so every rank learns which tokens failed);
5. tokens with a NaN row are reported in ``failed`` and their rows zeroed, so the caller can
   finish their requests with an error (the failed-input path) instead of running on garbage.

This follows the reference's compressed PLE embedding (vllm_sm80/models/qwen4_exp/exl3_ple.py:436
``Exl3PLEEmbedding``, row reader ``:180``, poison and masking ``:117-136``); the table layout is
``formats/ple.py``.  Without CUDA the decode runs on the fp32 oracle.
"""

from __future__ import annotations

import torch

from .. import _ext
from ..formats import ple as fple


class PleTable:
    def __init__(self, path: str, prefix: str, owner_lo: int = 0, owner_hi: int | None = None, *,
                 cache_rows: int | None = None, ways: int = 8, threads: int = 8, retries: int | None = None,
                 o_direct: bool = False, device=None, group=None):
        self.layout = lay = fple.read_layout(path, prefix)
        owner_hi = lay.rows if owner_hi is None else owner_hi
        if not 0 <= owner_lo <= owner_hi <= lay.rows:
            raise ValueError(f"owner range [{owner_lo}, {owner_hi}) outside the table's {lay.rows} rows")
        self.owner_lo, self.owner_hi = owner_lo, owner_hi
        self.dim, self.heads, self.bits = lay.dim, lay.heads, lay.bits
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.group = group
        from safetensors import safe_open

        with safe_open(path, framework="pt") as h:
            aux = {k: h.get_tensor(f"{prefix}.{k}") for k in fple.AUXILIARIES}
        self.head_bias = aux["head_bias"].to(self.device)
        self.head_offsets = aux["head_offsets"].to(self.device)
        self.head_vocab = aux["head_vocab_sizes"].to(self.device)
        self.layer_multipliers = aux["layer_multipliers"]
        self._offs_cpu, self._vocab_cpu = aux["head_offsets"], aux["head_vocab_sizes"]
        C = _ext.load()
        from .tables import storage_defaults

        cache_rows, retries = storage_defaults(lay.row_bytes, cache_rows, retries)
        self.reader = C.RowReader(path, lay.row_bytes, lay.rows, threads, retries, o_direct, lay.base)
        self.cache = C.RowCache(self.reader, cache_rows, ways)
        self._pinned = None
        self._copied = None  # the last host->device copy out of the pinned buffer

    def _host(self, n: int) -> torch.Tensor:
        if self._pinned is None or self._pinned.shape[0] < n:
            pin = self.device.type == "cuda"
            self._pinned = torch.empty(max(n, 64), self.layout.row_bytes, dtype=torch.uint8, pin_memory=pin)
        return self._pinned[:n]

    def _owned(self, ids: torch.Tensor) -> torch.Tensor:
        head = fple.head_of(ids, self._offs_cpu, self._vocab_cpu)
        return (head >= 0) & (ids >= self.owner_lo) & (ids < self.owner_hi)

    def read(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Host int16 [n, words] packed rows of the flat global ids and the uint8 failed-row flags
        (rows this rank does not own are zeros and never fail)."""
        ids = ids.reshape(-1).to("cpu", torch.int64)
        want = torch.where(self._owned(ids), ids, torch.full_like(ids, -1))
        if self._copied is not None:
            self._copied.synchronize()  # the previous lookup's copy still reads the pinned rows
            self._copied = None
        host = self._host(ids.numel())
        failed = self.cache.fetch(want, host)
        return host.view(torch.int16), failed

    def lookup(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """ids int64 [T, heads] -> (bf16 [T, heads*dim] on the table's device, bool [T] failed)."""
        T, H = ids.shape
        if H != self.heads:
            raise ValueError(f"ids have {H} heads, the table {self.heads}")
        flat = ids.reshape(-1).to("cpu", torch.int64)
        packed, failed = self.read(flat)
        if self.device.type == "cuda":
            rows = packed.to(self.device, non_blocking=True)
            fl = failed.to(self.device, non_blocking=True)
            dev_ids = flat.to(self.device, non_blocking=True)
            self._copied = torch.cuda.Event()
            self._copied.record()
            out = torch.empty(flat.numel(), self.dim, dtype=torch.bfloat16, device=self.device)
            _ext.ops().ple_decode(rows, dev_ids, self.head_bias, self.head_offsets, self.head_vocab,
                                  self.owner_lo, self.owner_hi, self.bits, fl, out)
        else:
            out = fple.decode_rows(packed, flat, self.head_bias, self.head_offsets, self.head_vocab,
                                   self.owner_lo, self.owner_hi, self.bits, failed)
        if self.group is not None:
            if out.is_cuda:
                torch.distributed.all_reduce(out, group=self.group)
            else:  # host backends may lack bf16 sums; the sum x + 0 + ... is exact in fp32
                f = out.float()
                torch.distributed.all_reduce(f, group=self.group)
                out = f.to(torch.bfloat16)
        out = out.view(T, H, self.dim)
        bad = out[..., 0].isnan().any(-1)
        out = out.reshape(T, H * self.dim).masked_fill(bad[:, None], 0)
        return out, bad

    def lookup_async(self, ids: torch.Tensor, fixed: bool = False) -> torch.Tensor:
        """Device ids [T, heads] -> bf16 [T, heads*dim] queued on the current stream with no host wait
        (the reference's host reader enqueued on the PLE stream, vllm_sm80/models/qwen4_exp/
        exl3_ple.py:829): the owned-id mask on the device, the ids' copy to pinned memory, the cache
        fetch as a host function, the rows' copy and the decode.  Failed reads come back as NaN rows
        (the caller masks them, e.g. with `mask_failed`).  fixed=True binds a job to this row count
        (CUDA-graph capture; run once outside capture first, with the largest count).  No tensor
        parallel sum here: the caller all-reduces the rows."""
        T, H = ids.shape
        n = T * H
        flat = ids.reshape(-1).to(torch.int64)
        offs, vocab = self.head_offsets, self.head_vocab
        h = torch.searchsorted(offs, flat, right=True) - 1
        hc = h.clamp_min(0)
        own = (h >= 0) & (flat - offs[hc] < vocab[hc]) & (flat >= self.owner_lo) & (flat < self.owner_hi)
        want = torch.where(own, flat, torch.full_like(flat, -1))
        st = self._staging(max(n, 64))
        stream = torch.cuda.current_stream(self.device)
        st["ids_h"][:n].copy_(want, non_blocking=True)
        args = (st["ids_h"].data_ptr(), n, st["rows_h"].data_ptr(), st["fail_h"].data_ptr())
        if fixed:
            job = st["jobs"].get(n)
            if job is None:
                job = st["jobs"][n] = self.cache.fixed_job(*args)
            self.cache.enqueue_job(stream.cuda_stream, job)
        else:
            self.cache.enqueue(stream.cuda_stream, *args)
        rows = st["rows_d"][:n]
        rows.copy_(st["rows_h"][:n], non_blocking=True)
        st["fail_d"][:n].copy_(st["fail_h"][:n], non_blocking=True)
        out = torch.empty(n, self.dim, dtype=torch.bfloat16, device=self.device)
        _ext.ops().ple_decode(rows.view(torch.int16), flat, self.head_bias, self.head_offsets, self.head_vocab,
                              self.owner_lo, self.owner_hi, self.bits, st["fail_d"][:n], out)
        return out.view(T, H * self.dim)

    @staticmethod
    def mask_failed(rows: torch.Tensor, heads: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Zero the tokens with a NaN row: (rows, failed [T]) without a host sync."""
        T = rows.shape[0]
        bad = rows.view(T, heads, -1)[..., 0].isnan().any(-1)
        return rows.masked_fill(bad[:, None], 0), bad

    def _staging(self, cap: int) -> dict:
        st = getattr(self, "_st", None)
        if st is None or st["cap"] < cap:
            if st is not None and st["jobs"]:
                raise RuntimeError("the staging of captured lookups cannot grow; make the first lookup the largest")
            rb = self.layout.row_bytes
            dev = self.device
            st = self._st = dict(cap=cap, jobs={},
                                 ids_h=torch.empty(cap, dtype=torch.int64, pin_memory=True),
                                 rows_h=torch.empty(cap, rb, dtype=torch.uint8, pin_memory=True),
                                 fail_h=torch.empty(cap, dtype=torch.uint8, pin_memory=True),
                                 rows_d=torch.empty(cap, rb, dtype=torch.uint8, device=dev),
                                 fail_d=torch.empty(cap, dtype=torch.uint8, device=dev))
        return st

    def stats(self) -> dict:
        r = self.reader.stats()
        h = self.cache.stats()
        return {"reads": r[0], "retries": r[1], "failures": r[2], "bytes": r[3], "hits": h[0], "misses": h[1]}
