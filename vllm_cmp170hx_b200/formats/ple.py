"""EXL3-coded per-layer-embedding (PLE) tables: file layout, writer and fp32 oracle decode.

A table is a safetensors file (the layout of the reference's compressed n-gram tables,
vllm_sm80/kernels/exl3/utils.py:324, kept alike so existing table files load) holding, under one
prefix:

* ``{prefix}.trellis`` int16 ``[rows, 1 + dim*K/16]``: per row an fp16 scale word, then a
  tail-biting ring of ``dim*K`` bits (bit i in word i/16 at position i%16; channel c owns ring
  bits ``[c*K, (c+1)*K)``);
* ``{prefix}.head_bias`` fp16 ``[heads, dim]``; ``{prefix}.head_offsets`` / ``head_vocab_sizes``
  int64 ``[heads]`` (contiguous heads from row 0, fewer than 128 padding rows after the last);
  ``{prefix}.layer_multipliers`` int64 (the n-gram hash multipliers, for the caller);
* metadata ``format=exl3_ngram_trellis``, ``version=1``, ``codebook=mul1``, ``K``, ``row_dim``, ``rows``.

Decoding channel c of a row: the 16-bit state takes channel c's K bits as its low field and the
fields of channels c-1, c-2, ... (mod dim) above them; the EXL3 "mul1" codebook maps it to
fp16(fp16(1024 + bytesum(state * 0x83DCD12D)) * a + b) with a, b the fp16 words 0x1eee, 0xc931;
then value * scale (fp32) + bias (fp32) rounded to bf16.  Ids outside the caller's owner range or
every head's vocabulary decode to zero rows; a NaN scale (a row the host failed to read) gives a
NaN row.  ``decode_rows`` is the oracle of ``csrc/rows.cu::ple_decode_kernel`` (the reference's
kernel is csrc/exl3/ple.cu:91).
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import torch

FORMAT = "exl3_ngram_trellis"
AUXILIARIES = ("head_bias", "head_offsets", "head_vocab_sizes", "layer_multipliers")
POISON_SCALE = 0x7E00  # an fp16 quiet NaN
_A, _B = 0x1EEE, 0xC931
_MULT = 0x83DCD12D


def words_per_row(dim: int, bits: int) -> int:
    if not 1 <= bits <= 16 or dim <= 0 or dim * bits % 16:
        raise ValueError(f"{dim} channels at K={bits} do not fill whole 16-bit words")
    return 1 + dim * bits // 16


def _half(bits: int) -> torch.Tensor:
    return torch.tensor([bits], dtype=torch.int32).to(torch.int16).view(torch.float16)


def codebook_value(state: torch.Tensor) -> torch.Tensor:
    """mul1 codebook: int64 states in [0, 2^16) -> fp16 values."""
    p = (state.to(torch.int64) * _MULT) & 0xFFFFFFFF
    s = (p & 255) + ((p >> 8) & 255) + ((p >> 16) & 255) + (p >> 24)
    a, b = _half(_A).float(), _half(_B).float()
    # the product is exact in fp32 and so is the sum; one rounding to fp16
    return ((1024 + s).float() * a + b).half()


def ring_states(trellis: torch.Tensor, dim: int, bits: int) -> torch.Tensor:
    """int16 [n, words] -> int64 [n, dim] trellis states."""
    n = trellis.shape[0]
    w = trellis[:, 1:].to(torch.int64) & 0xFFFF
    ring = ((w.unsqueeze(-1) >> torch.arange(16)) & 1).reshape(n, -1)
    c = torch.arange(dim)[:, None]
    m = torch.arange(16)[None]
    src = ((c - m // bits) % dim) * bits + m % bits
    return (ring[:, src] << m).sum(-1)


def head_of(ids: torch.Tensor, offsets: torch.Tensor, vocab: torch.Tensor) -> torch.Tensor:
    """The head of each id, or -1 where no head's vocabulary holds it."""
    h = torch.searchsorted(offsets, ids, right=True) - 1
    hc = h.clamp_min(0)
    ok = (h >= 0) & (ids - offsets[hc] < vocab[hc]) & (vocab[hc] > 0)
    return torch.where(ok, h, torch.full_like(h, -1))


def decode_rows(trellis: torch.Tensor, ids: torch.Tensor, head_bias: torch.Tensor, head_offsets: torch.Tensor,
                head_vocab: torch.Tensor, owner_lo: int, owner_hi: int, bits: int,
                failed: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 oracle: packed rows int16 [n, words] of global ids [n] -> bf16 [n, dim]."""
    trellis, ids = trellis.cpu(), ids.cpu().to(torch.int64)
    head_bias = head_bias.cpu()
    dim = head_bias.shape[1]
    words_per_row(dim, bits)
    head = head_of(ids, head_offsets.cpu(), head_vocab.cpu())
    head = torch.where((ids >= owner_lo) & (ids < owner_hi), head, torch.full_like(head, -1))
    v = codebook_value(ring_states(trellis, dim, bits)).float()
    scale = (trellis[:, 0].contiguous().view(torch.float16)).float()
    if failed is not None:
        scale = torch.where(failed.cpu().bool(), torch.full_like(scale, float("nan")), scale)
    bias = head_bias[head.clamp_min(0)].float()
    y = (v * scale[:, None] + bias).to(torch.bfloat16)
    return torch.where((head >= 0)[:, None], y, torch.zeros_like(y))


def random_table(heads: int, vocab: int, dim: int, bits: int, seed: int = 0, padding: int = 0):
    """A synthetic table: random rings, scales in [0.01, 0.1), biases in [-0.05, 0.05)."""
    g = torch.Generator().manual_seed(seed)
    rows = heads * vocab + padding
    words = words_per_row(dim, bits)
    trellis = torch.randint(-32768, 32768, (rows, words), generator=g, dtype=torch.int32).to(torch.int16)
    scale = (0.01 + 0.09 * torch.rand(rows, generator=g)).half()
    trellis[:, 0] = scale.view(torch.int16)
    return {
        "trellis": trellis,
        "head_bias": ((torch.rand(heads, dim, generator=g) - 0.5) * 0.1).half(),
        "head_offsets": torch.arange(heads, dtype=torch.int64) * vocab,
        "head_vocab_sizes": torch.full((heads,), vocab, dtype=torch.int64),
        "layer_multipliers": torch.randint(1, 1 << 30, (4,), generator=g, dtype=torch.int64),
    }


def write_table(path: str, prefix: str, table: dict, bits: int) -> None:
    from safetensors.torch import save_file

    rows, dim = table["trellis"].shape[0], table["head_bias"].shape[1]
    meta = {"format": FORMAT, "version": "1", "codebook": "mul1", "K": str(bits), "row_dim": str(dim),
            "rows": str(rows)}
    save_file({f"{prefix}.{k}": v.contiguous() for k, v in table.items()}, path, metadata=meta)


@dataclass(frozen=True)
class Layout:
    """Geometry of one table file: where the trellis rows start and how they are cut."""

    path: str
    prefix: str
    base: int  # byte offset of row 0 of the trellis in the file
    rows: int
    words: int
    bits: int
    dim: int
    heads: int
    head_offsets: tuple[int, ...]
    head_vocab_sizes: tuple[int, ...]

    @property
    def row_bytes(self) -> int:
        return 2 * self.words


def read_layout(path: str, prefix: str) -> Layout:
    """Parse and validate a table file's header (safetensors: u64 header length, JSON header, data)."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
    meta = header.get("__metadata__", {})
    if meta.get("format") != FORMAT or meta.get("version") != "1" or meta.get("codebook") != "mul1":
        raise ValueError(f"{path}: not an EXL3 n-gram trellis table")
    tr, bias = header.get(prefix + ".trellis"), header.get(prefix + ".head_bias")
    if tr is None or tr["dtype"] != "I16" or len(tr["shape"]) != 2:
        raise ValueError(f"{path}: {prefix}.trellis missing or not int16 [rows, words]")
    if bias is None or bias["dtype"] != "F16" or len(bias["shape"]) != 2:
        raise ValueError(f"{path}: {prefix}.head_bias missing or not fp16 [heads, dim]")
    rows, words = tr["shape"]
    heads, dim = bias["shape"]
    bits = int(meta.get("K", "0"))
    if heads <= 0 or words != words_per_row(dim, bits):
        raise ValueError(f"{path}: rows of {words} words do not hold {dim} channels at K={bits}")
    if int(meta.get("row_dim", -1)) != dim or int(meta.get("rows", -1)) != rows:
        raise ValueError(f"{path}: metadata disagrees with the tensor headers")
    from safetensors import safe_open

    with safe_open(path, framework="pt") as h:
        offs = h.get_tensor(prefix + ".head_offsets").tolist()
        sizes = h.get_tensor(prefix + ".head_vocab_sizes").tolist()
    if len(offs) != heads or len(sizes) != heads:
        raise ValueError(f"{path}: head tables are not [heads]")
    end = 0
    for o, s in zip(offs, sizes):
        if o != end or s <= 0:
            raise ValueError(f"{path}: heads are not contiguous from row 0")
        end += s
    if end > rows or rows - end >= 128:
        raise ValueError(f"{path}: {rows - end} padding rows after the heads")
    base = 8 + hlen + tr["data_offsets"][0]
    return Layout(path, prefix, base, rows, words, bits, dim, heads, tuple(offs), tuple(sizes))
