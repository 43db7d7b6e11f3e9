"""Engram n-gram memory of the DeepSeek-V4.1-style model (the reference's Engram embedding,
vllm_sm80/models/deepseek_v41/sm80_engram.py:879, storage of :562; its gated block is the upstream
module that embedding feeds).

* :class:`EngramMemory` -- one storage-backed table (storage/tables.py: e4m3 rows with E8M0 block
  scales, host LRU row cache, threaded reads with retries, GPU dequant) of ``engram_heads`` hash heads x
  ``engram_vocab`` rows; head h hashes the last ``engram_orders[h]`` tokens (models/qwen.py::ngram_ids
  with this table's multipliers).  The step's ids are computed on the host with the other step inputs;
  one lookup per step (queued on the stream, CUDA-graph capturable) serves every Engram layer.
* :class:`EngramBlock` -- per Engram layer: ``[k | v] = rows W^T`` (one GEMM), the gate
  ``alpha = sigmoid(<rmsnorm(h) w_h, rmsnorm(k) w_k> / sqrt(H))`` and ``a += alpha v`` into the layer's
  attention output (csrc/engram.cu), h being the layer's normalised input.

A row the host failed to read dequantises to NaN, so only the tokens (and requests) that used it turn
NaN and finish through the failed-input path.
"""

from __future__ import annotations

import os
import tempfile

import numpy as np
import torch
from torch import nn

from .. import _ext
from ..config import ModelConfig
from .layers import Linear, WeightInit, default_std
from .qwen import ngram_ids

# hash multipliers of the synthetic tables (odd 32-bit constants)
_MULT = np.array([0x9E3779B1, 0x85EBCA77, 0xC2B2AE3D, 0x27D4EB2F, 0x165667B1, 0xD3A2646C], dtype=np.int64)


class EngramMemory:
    def __init__(self, cfg: ModelConfig, device, seed: int = 0):
        from ..storage import tables

        self.heads, self.dim, self.vocab = cfg.engram_heads, cfg.engram_dim, cfg.engram_vocab
        if self.dim % 256:
            raise ValueError("engram_dim must be a multiple of 256 (E8M0 blocks of 32, 8-byte rows)")
        rows = self.heads * self.vocab
        path = cfg.engram_path
        if not path:
            d = tempfile.mkdtemp(prefix="b200_engram_")
            path = os.path.join(d, "engram.bin")
            g = torch.Generator().manual_seed(seed + 5151)
            tables.write_table(path, torch.randn(rows, self.dim, generator=g) * 0.5)
        self.path = path
        self.table = tables.RowTable(path, rows, self.dim, device=device)
        self.device = torch.device(device)
        self.orders = list(cfg.engram_orders) or [2] * self.heads
        if len(self.orders) != self.heads:
            raise ValueError("engram_orders needs one n-gram order per Engram head")
        self.max_order = max(self.orders)
        self.offsets = np.arange(self.heads, dtype=np.int64) * self.vocab
        self.vocab_sizes = np.full(self.heads, self.vocab, dtype=np.int64)

    def ids_of(self, tokens, positions: np.ndarray) -> np.ndarray:
        return ngram_ids(np.asarray(tokens, dtype=np.int64), positions, self.orders, self.offsets, self.vocab_sizes,
                         _MULT)

    def reserve(self, max_tokens: int) -> None:
        if self.device.type == "cuda":
            self.table._staging(max(max_tokens, 64) * self.heads)

    def rows(self, ids: torch.Tensor) -> torch.Tensor:
        """ids int64 [T, heads] -> [T, heads * dim] bf16 (NaN rows for failed reads)."""
        T = ids.shape[0]
        if ids.is_cuda:
            out = self.table.lookup_async(ids, fixed=torch.cuda.is_current_stream_capturing())
        else:
            out = self.table.lookup(ids)
        return out.view(T, self.heads * self.dim)

    _streams: dict = {}

    def prefetch(self, ids: torch.Tensor):
        """Start the step's lookup on a side stream (the reference's Engram prefetch on its own stream,
        vllm_sm80/models/deepseek_v41/sm80_engram_prefetch.py): the ids' copy out, the host fetch, the rows'
        copy in and the dequant run beside the layers before the first Engram layer.  Returns (rows,
        event); a consumer waits for the event before reading the rows.  On CPU: (rows, None)."""
        if not ids.is_cuda:
            return self.rows(ids), None
        dev = ids.device
        side = EngramMemory._streams.get(dev)
        if side is None:
            side = EngramMemory._streams[dev] = torch.cuda.Stream(dev)
        cur = torch.cuda.current_stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            rows = self.rows(ids)
            ev = torch.cuda.Event()
            ev.record(side)
        if not torch.cuda.is_current_stream_capturing():  # graph buffers live as long as the graph
            ids.record_stream(side)
            rows.record_stream(cur)
        return rows, ev


class EngramBlock(nn.Module):
    def __init__(self, cfg: ModelConfig, wi: WeightInit):
        super().__init__()
        H = cfg.hidden_size
        width = cfg.engram_heads * cfg.engram_dim
        self.kv = Linear(wi.normal((2 * H, width), default_std(width)))
        self.h_norm_w = nn.Parameter(wi.ones_plus(H, 0.05), requires_grad=False)
        self.k_norm_w = nn.Parameter(wi.ones_plus(H, 0.05), requires_grad=False)
        self.eps = cfg.rms_eps

    def add_(self, a: torch.Tensor, h: torch.Tensor, rows: torch.Tensor, ready=None) -> torch.Tensor:
        """a += sigmoid(<rmsnorm(h) w_h, rmsnorm(k) w_k> / sqrt(H)) v, [k | v] = rows W^T; returns a.
        ready: the prefetch's event (waited for on the current stream before the rows are read)."""
        if ready is not None:
            torch.cuda.current_stream(rows.device).wait_event(ready)
        kv = self.kv(rows)
        if a.is_cuda:
            _ext.ops().engram_gate(h, kv, self.h_norm_w, self.k_norm_w, self.eps, a)
            return a
        return a.copy_(gate_ref(a, h, kv, self.h_norm_w, self.k_norm_w, self.eps))


def gate_ref(a, h, kv, wh, wk, eps):
    """fp32 definition of the Engram gate (the CPU path and the GPU test's oracle)."""
    H = h.shape[1]
    hf, k, v = h.float(), kv[:, :H].float(), kv[:, H:2 * H].float()
    hn = hf * torch.rsqrt((hf * hf).mean(-1, keepdim=True) + eps) * wh.float()
    kn = k * torch.rsqrt((k * k).mean(-1, keepdim=True) + eps) * wk.float()
    alpha = torch.sigmoid((hn * kn).sum(-1, keepdim=True) / H ** 0.5)
    return (a.float() + alpha * v).to(a.dtype)
