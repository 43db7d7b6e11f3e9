"""Embedding tables whose rows live in a file and are fetched per step.

``RowTable(path, num_rows, dim)`` serves ``lookup(ids) -> bf16 [n, dim]``:

1. the native ``RowCache`` (``csrc/row_store.cpp``) copies cached rows and
   reads the misses from the file on a thread pool (retries with a 1 ms
   doubling backoff, then the row is reported failed) into a pinned buffer;
2. one asynchronous host->device copy;
3. the dequant kernel (``csrc/rows.cu``) turns e4m3 codes with E8M0 block
   scales into bf16 and writes NaN for failed rows, so the failed-input path
   finishes exactly the requests that used them.

File format: ``num_rows`` rows of ``dim`` e4m3 bytes followed by ``dim / 32``
E8M0 scale bytes, padded to 8 bytes (``write_table`` produces it).  This is
the row format of the DeepSeek-V4.1 Engram tables in the reference
(E4M3 x E8M0, models/deepseek_v41/ops/sm80_engram_dequant.py); its PLE tables
are EXL3-coded instead, which this module does not read.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _ext


def row_bytes(dim: int) -> int:
    return (dim + dim // 32 + 7) // 8 * 8


def quantize_rows(x: torch.Tensor) -> np.ndarray:
    """fp32 [n, dim] -> uint8 [n, row_bytes]: e4m3 codes with one E8M0 (power-of-two) scale per 32."""
    n, d = x.shape
    assert d % 256 == 0
    blocks = x.float().view(n, d // 32, 32)
    amax = blocks.abs().amax(-1).clamp_min(1e-30)
    e = torch.ceil(torch.log2(amax / 448.0)).clamp(-127, 127)
    q = (blocks / torch.exp2(e)[..., None]).to(torch.float8_e4m3fn).view(torch.uint8).view(n, d)
    out = np.zeros((n, row_bytes(d)), dtype=np.uint8)
    out[:, :d] = q.numpy()
    out[:, d:d + d // 32] = (e + 127).to(torch.uint8).numpy()
    return out


def dequantize_rows(raw: torch.Tensor, dim: int) -> torch.Tensor:
    """Reference dequantisation (CPU): uint8 [n, row_bytes] -> fp32 [n, dim]."""
    codes = raw[:, :dim].contiguous().view(torch.float8_e4m3fn).float()
    e = raw[:, dim:dim + dim // 32].float() - 127.0
    return (codes.view(-1, dim // 32, 32) * torch.exp2(e)[..., None]).view(-1, dim)


def write_table(path: str, x: torch.Tensor) -> None:
    quantize_rows(x).tofile(path)


def storage_defaults(row_bytes: int, cache_rows: int | None, retries: int | None) -> tuple[int, int]:
    """Host-cache rows and read retries of a storage-backed table: the arguments when given, else
    VLLM_B200_ROW_CACHE_GIB worth of rows (0: 65536 rows) and VLLM_B200_PLE_READ_RETRIES."""
    from .. import envs

    if cache_rows is None:
        gib = envs.get("VLLM_B200_ROW_CACHE_GIB")
        cache_rows = max(1024, int(gib * (1 << 30)) // max(1, row_bytes)) if gib > 0 else 1 << 16
    if retries is None:
        retries = envs.get("VLLM_B200_PLE_READ_RETRIES")
    return cache_rows, retries


class RowTable:
    def __init__(self, path: str, num_rows: int, dim: int, cache_rows: int | None = None, ways: int = 8,
                 threads: int = 8, retries: int | None = None, o_direct: bool = False, device=None):
        """cache_rows / retries default to VLLM_B200_ROW_CACHE_GIB (as rows; 0: 65536 rows) and
        VLLM_B200_PLE_READ_RETRIES."""
        C = _ext.load()
        self.dim = dim
        self.row_bytes = row_bytes(dim)
        cache_rows, retries = storage_defaults(self.row_bytes, cache_rows, retries)
        self.reader = C.RowReader(path, self.row_bytes, num_rows, threads, retries, o_direct)
        self.cache = C.RowCache(self.reader, cache_rows, ways)
        self.device = torch.device(device) if device is not None else None
        self._pinned = None
        self._copied = None  # the last host->device copy out of the pinned buffer
        self._st = None  # staging of the stream-ordered lookup

    def _host(self, n: int) -> torch.Tensor:
        if self._pinned is None or self._pinned.shape[0] < n:
            pin = self.device is not None and self.device.type == "cuda"
            self._pinned = torch.empty(max(n, 64), self.row_bytes, dtype=torch.uint8, pin_memory=pin)
        return self._pinned[:n]

    def lookup(self, ids: torch.Tensor) -> torch.Tensor:
        """bf16 [n, dim] rows of `ids`; rows whose read failed are NaN."""
        ids = ids.reshape(-1).to("cpu", torch.int64)
        if self._copied is not None:
            self._copied.synchronize()  # the previous lookup's copy still reads the pinned rows
            self._copied = None
        host = self._host(ids.numel())
        failed = self.cache.fetch(ids, host)
        if self.device is None or self.device.type != "cuda":
            out = dequantize_rows(host, self.dim)
            out[failed.bool()] = float("nan")
            return out.to(torch.bfloat16)
        raw = host.to(self.device, non_blocking=True)
        fl = failed.to(self.device, non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record()
        out = torch.empty(ids.numel(), self.dim, dtype=torch.bfloat16, device=self.device)
        _ext.ops().dequant_rows(raw, self.dim, fl, out)
        return out

    def _staging(self, cap: int) -> dict:
        if self._st is None or self._st["cap"] < cap:
            if self._st is not None and self._st["jobs"]:
                raise RuntimeError("the staging of captured lookups cannot grow; make the first lookup the largest")
            dev = self.device
            self._st = dict(cap=cap, jobs={},
                            ids_h=torch.empty(cap, dtype=torch.int64, pin_memory=True),
                            rows_h=torch.empty(cap, self.row_bytes, dtype=torch.uint8, pin_memory=True),
                            fail_h=torch.empty(cap, dtype=torch.uint8, pin_memory=True),
                            rows_d=torch.empty(cap, self.row_bytes, dtype=torch.uint8, device=dev),
                            fail_d=torch.empty(cap, dtype=torch.uint8, device=dev))
        return self._st

    def lookup_async(self, ids: torch.Tensor, fixed: bool = False) -> torch.Tensor:
        """bf16 [n, dim] rows of the device ids [n] queued on the current stream with no host wait: the
        ids' copy to pinned memory, the cache fetch as a host function (the reference's host-function
        readers, csrc/exl3/ple_read.cpp:179 run_queued, csrc/exl3/engram_fetch.cpp:454 execute_fixed),
        the rows' copy to the device and the dequant.  Calls share one staging and must stay on one
        stream.  fixed=True binds a job to this row count and the staging, so the lookup can be
        captured in a CUDA graph (each replay fetches that replay's ids); run it once outside capture
        first, with the largest count, so the staging exists."""
        n = ids.numel()
        st = self._staging(max(n, 64))
        stream = torch.cuda.current_stream(self.device)
        st["ids_h"][:n].copy_(ids.reshape(-1).to(torch.int64), non_blocking=True)
        args = (st["ids_h"].data_ptr(), n, st["rows_h"].data_ptr(), st["fail_h"].data_ptr())
        if fixed:
            job = st["jobs"].get(n)
            if job is None:
                job = st["jobs"][n] = self.cache.fixed_job(*args)
            self.cache.enqueue_job(stream.cuda_stream, job)
        else:
            self.cache.enqueue(stream.cuda_stream, *args)
        st["rows_d"][:n].copy_(st["rows_h"][:n], non_blocking=True)
        st["fail_d"][:n].copy_(st["fail_h"][:n], non_blocking=True)
        out = torch.empty(n, self.dim, dtype=torch.bfloat16, device=self.device)
        _ext.ops().dequant_rows(st["rows_d"][:n], self.dim, st["fail_d"][:n], out)
        return out
