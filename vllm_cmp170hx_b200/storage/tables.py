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


class RowTable:
    def __init__(self, path: str, num_rows: int, dim: int, cache_rows: int = 1 << 16, ways: int = 8,
                 threads: int = 8, retries: int = 3, o_direct: bool = False, device=None):
        C = _ext.load()
        self.dim = dim
        self.row_bytes = row_bytes(dim)
        self.reader = C.RowReader(path, self.row_bytes, num_rows, threads, retries, o_direct)
        self.cache = C.RowCache(self.reader, cache_rows, ways)
        self.device = torch.device(device) if device is not None else None
        self._pinned = None

    def _host(self, n: int) -> torch.Tensor:
        if self._pinned is None or self._pinned.shape[0] < n:
            pin = self.device is not None and self.device.type == "cuda"
            self._pinned = torch.empty(max(n, 64), self.row_bytes, dtype=torch.uint8, pin_memory=pin)
        return self._pinned[:n]

    def lookup(self, ids: torch.Tensor) -> torch.Tensor:
        """bf16 [n, dim] rows of `ids`; rows whose read failed are NaN."""
        ids = ids.reshape(-1).to("cpu", torch.int64)
        host = self._host(ids.numel())
        failed = self.cache.fetch(ids, host)
        if self.device is None or self.device.type != "cuda":
            out = dequantize_rows(host, self.dim)
            out[failed.bool()] = float("nan")
            return out.to(torch.bfloat16)
        raw = host.to(self.device, non_blocking=True)
        fl = failed.to(self.device, non_blocking=True)
        out = torch.empty(ids.numel(), self.dim, dtype=torch.bfloat16, device=self.device)
        _ext.ops().dequant_rows(raw, self.dim, fl, out)
        return out
