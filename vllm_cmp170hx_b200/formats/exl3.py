"""EXL3 trellis-quantised matrices: checkpoint layout, CPU decoder, random init.

Checkpoint tensors of one matrix ``<prefix>`` (the layout the reference's
loader accepts, vllm_sm80/kernels/exl3/utils.py:124-290):

* ``<prefix>.trellis``  int16 ``[K/16, N/16, 8*bits_x2]`` (K = padded_in,
  N = padded_out, both multiples of 128);
* ``<prefix>.suh`` fp16 ``[K]`` and ``<prefix>.svh`` fp16 ``[N]`` (input /
  output sign-and-scale vectors around the Hadamard rotations);
* one int32 scalar marker naming the codebook: ``mcg`` (codebook 1) or
  ``mul1`` (codebook 2), holding that codebook's multiplier.

Math (csrc/exl3/reference.cu:20-200 of the reference):
``y = H128( H128(x * suh) @ W ) * svh`` where H128 is the normalised
Sylvester Hadamard transform applied to every 128-block of the last axis and
W[k, n] is decoded from a 16-bit window of the tile's bit ring:

* 16x16 tile (k // 16, n // 16), r = k % 16, c = n % 16;
* lane = (c & 7) * 4 + ((r & 7) >> 1);  idx = lane*8 + (r & 1) + 2*(r >> 3) + 4*(c >> 3);
* end = (idx+1) * (bits_x2 // 2) + ((idx+1) // 2 if bits_x2 is odd);
  start = (end - 16) mod (128 * bits_x2);
* the tile's int16 pairs form uint32 ring words (word w = e[2w] | e[2w+1] << 16)
  read most-significant bit first; the state is the 16 bits at ``start``.
* codebook 1: p = s * 0xCBAC1FED; p = (p & 0x8FFF8FFF) ^ 0x3B603B60;
  value = fp16(p & 0xFFFF) + fp16(p >> 16)  (fp16 add);
  codebook 2: p = s * 0x83DCD12D; t = sum of p's four bytes;
  value = fma16(fp16 bits 0x6400 + t, fp16 bits 0x1EEE, fp16 bits 0xC931).

These constants are the EXL3 format's own (MIT-licensed exllamav3 format);
a decoder of that checkpoint format cannot choose different ones.
"""

from __future__ import annotations

import dataclasses
import math

import torch

MCG_MULT = 0xCBAC1FED
MUL1_MULT = 0x83DCD12D
MARKERS = {"mcg": (1, MCG_MULT), "mul1": (2, MUL1_MULT)}
H128_SCALE = 1.0 / math.sqrt(128.0)


def supported(bits_x2: int, codebook: int) -> bool:
    return bits_x2 in range(2, 17, 2) or (codebook == 2 and bits_x2 in (3, 5, 7))


@dataclasses.dataclass
class Exl3Matrix:
    """One EXL3 matrix. ``in_features``/``out_features`` are the logical sizes
    (<= padded K/N); inputs are zero-padded, outputs truncated."""

    trellis: torch.Tensor  # int16 [K/16, N/16, 8*bits_x2]
    suh: torch.Tensor  # fp16 [K]
    svh: torch.Tensor  # fp16 [N]
    bits_x2: int
    codebook: int
    in_features: int
    out_features: int

    @property
    def padded_in(self) -> int:
        return self.trellis.shape[0] * 16

    @property
    def padded_out(self) -> int:
        return self.trellis.shape[1] * 16

    def to(self, device) -> "Exl3Matrix":
        return dataclasses.replace(self, trellis=self.trellis.to(device), suh=self.suh.to(device),
                                   svh=self.svh.to(device))

    def state_dict(self, prefix: str) -> dict[str, torch.Tensor]:
        marker = "mcg" if self.codebook == 1 else "mul1"
        mult = MARKERS[marker][1]
        return {
            f"{prefix}.trellis": self.trellis,
            f"{prefix}.suh": self.suh,
            f"{prefix}.svh": self.svh,
            f"{prefix}.{marker}": torch.tensor(mult - (1 << 32) if mult >= 1 << 31 else mult, dtype=torch.int32),
        }

    @staticmethod
    def from_state_dict(sd: dict[str, torch.Tensor], prefix: str, in_features: int | None = None,
                        out_features: int | None = None) -> "Exl3Matrix":
        trellis = sd[f"{prefix}.trellis"]
        if trellis.dtype != torch.int16 or trellis.dim() != 3 or trellis.shape[2] % 8:
            raise ValueError(f"invalid EXL3 trellis: {prefix}")
        K, N = trellis.shape[0] * 16, trellis.shape[1] * 16
        if K % 128 or N % 128:
            raise ValueError(f"invalid EXL3 tile geometry: {prefix}")
        markers = [m for m in MARKERS if f"{prefix}.{m}" in sd]
        if len(markers) != 1:
            raise ValueError(f"missing or conflicting EXL3 codebook marker: {prefix}")
        codebook, mult = MARKERS[markers[0]]
        if int(sd[f"{prefix}.{markers[0]}"].item()) & 0xFFFFFFFF != mult:
            raise ValueError(f"unsupported EXL3 codebook multiplier: {prefix}")
        bits_x2 = trellis.shape[2] // 8
        if not supported(bits_x2, codebook):
            raise ValueError(f"unsupported EXL3 bitrate/codebook: {prefix}")
        suh, svh = sd[f"{prefix}.suh"], sd[f"{prefix}.svh"]
        if suh.shape != (K,) or svh.shape != (N,):
            raise ValueError(f"EXL3 suh/svh geometry mismatch: {prefix}")
        return Exl3Matrix(trellis, suh, svh, bits_x2, codebook, in_features or K, out_features or N)


# ----------------------------------------------------------------------------- codebooks
def _u32(x: torch.Tensor) -> torch.Tensor:
    return x & 0xFFFFFFFF


def _f16_from_bits(bits: torch.Tensor) -> torch.Tensor:
    b = bits.to(torch.int32)
    b = torch.where(b >= 32768, b - 65536, b).to(torch.int16)
    return b.view(torch.float16)


def codebook_value(state: torch.Tensor, codebook: int) -> torch.Tensor:
    """fp16 value of 16-bit trellis states (int64 tensor), exactly as the format defines it."""
    s = state.to(torch.int64)
    if codebook == 1:
        p = _u32(s * MCG_MULT)
        p = (p & 0x8FFF8FFF) ^ 0x3B603B60
        lo, hi = _f16_from_bits(p & 0xFFFF), _f16_from_bits(p >> 16)
        return (lo.double() + hi.double()).to(torch.float16)  # one rounding, as fp16 add
    p = _u32(s * MUL1_MULT)
    t = (p & 255) + ((p >> 8) & 255) + ((p >> 16) & 255) + (p >> 24)
    a = _f16_from_bits(0x6400 + t).float()
    b = _f16_from_bits(torch.full_like(t, 0x1EEE)).float()
    c = _f16_from_bits(torch.full_like(t, 0xC931)).float()
    # fp16 fma rounds once: the fp32 product of two fp16 values is exact, and
    # the fp32 sum of that product and c is rounded then re-rounded to fp16.
    # Doing the sum in float64 keeps it exact before the single fp16 rounding.
    return (a.double() * b.double() + c.double()).to(torch.float16)


def _tile_geometry(bits_x2: int, device=None):
    """Per in-tile position (r, c) -> (word index lo, bit offset) of its state."""
    r = torch.arange(16, device=device).view(16, 1).expand(16, 16)
    c = torch.arange(16, device=device).view(1, 16).expand(16, 16)
    lane = (c & 7) * 4 + ((r & 7) >> 1)
    idx = lane * 8 + (r & 1) + 2 * (r >> 3) + 4 * (c >> 3)
    whole = bits_x2 // 2
    end = (idx + 1) * whole + (((idx + 1) // 2) if bits_x2 & 1 else 0)
    ring = 128 * bits_x2
    start = (end - 16 + ring) % ring
    return start  # [16, 16]


def decode_weight(trellis: torch.Tensor, bits_x2: int, codebook: int) -> torch.Tensor:
    """Full fp16 weight [K, N] of a trellis [K/16, N/16, 8*bits_x2] (CPU/GPU torch, vectorised)."""
    kt, nt, stride = trellis.shape
    words_n = stride // 2
    e = trellis.to(torch.int64) & 0xFFFF
    words = e[..., 0::2] | (e[..., 1::2] << 16)  # [kt, nt, words_n] uint32 in int64
    start = _tile_geometry(bits_x2, trellis.device)  # [16, 16]
    lo = start // 32
    hi = (lo + 1) % words_n
    wa = words[:, :, lo.flatten()].view(kt, nt, 16, 16)
    wb = words[:, :, hi.flatten()].view(kt, nt, 16, 16)
    # state = bits [off, off+16) of the 64-bit window (wa:wb), MSB first.
    off = (start & 31).view(1, 1, 16, 16)
    left = (wa >> (16 - off).clamp(min=0)) & 0xFFFF
    right = ((wa << (off - 16).clamp(min=0)) | (wb >> (48 - off).clamp(max=32))) & 0xFFFF
    state = torch.where(off <= 16, left, right)
    vals = codebook_value(state, codebook)  # [kt, nt, 16(r), 16(c)]
    return vals.permute(0, 2, 1, 3).reshape(kt * 16, nt * 16)


def hadamard128(x: torch.Tensor) -> torch.Tensor:
    """Normalised Sylvester H128 on every 128-block of the last axis (fp32)."""
    shape = x.shape
    y = x.float().reshape(-1, shape[-1] // 128, 128)
    d = 1
    while d < 128:
        y = y.view(*y.shape[:-1], 128 // (2 * d), 2, d)
        a, b = y[..., 0, :], y[..., 1, :]
        y = torch.stack((a + b, a - b), dim=-2).reshape(*y.shape[:-3], 128)
        d *= 2
    return (y * H128_SCALE).reshape(shape)


def linear(x: torch.Tensor, m: Exl3Matrix, weight: torch.Tensor | None = None) -> torch.Tensor:
    """Reference EXL3 linear in fp32: y = H128(H128(x*suh) @ W) * svh (logical sizes)."""
    K, N = m.padded_in, m.padded_out
    xf = torch.zeros(*x.shape[:-1], K, dtype=torch.float32, device=x.device)
    xf[..., : m.in_features] = x.float()
    xt = hadamard128(xf * m.suh.float())
    W = weight if weight is not None else decode_weight(m.trellis, m.bits_x2, m.codebook).float()
    y = hadamard128(xt @ W) * m.svh.float()
    return y[..., : m.out_features]


def random_matrix(in_features: int, out_features: int, bits_x2: int = 8, codebook: int = 2,
                  generator: torch.Generator | None = None, device="cpu", out_scale: float = 1.0) -> Exl3Matrix:
    """Random-init EXL3 matrix: every 16-bit trellis state is a valid code, suh = +-1,
    svh = +-out_scale/sqrt(K) so the output variance matches a unit-variance
    dense layer's (the codebook's values have unit variance)."""
    K = (in_features + 127) // 128 * 128
    N = (out_features + 127) // 128 * 128
    g = generator
    trellis = torch.randint(-32768, 32768, (K // 16, N // 16, 8 * bits_x2), dtype=torch.int32, generator=g)
    trellis = trellis.to(torch.int16)
    sgn = lambda n: (torch.randint(0, 2, (n,), generator=g) * 2 - 1).to(torch.float32)  # noqa: E731
    suh = sgn(K).to(torch.float16)
    svh = (sgn(N) * (out_scale / math.sqrt(K))).to(torch.float16)
    return Exl3Matrix(trellis.to(device), suh.to(device), svh.to(device), bits_x2, codebook, in_features,
                      out_features)


def stack_experts(mats: list[Exl3Matrix]) -> dict[str, torch.Tensor]:
    """Contiguous per-expert buffers (one allocation per tensor kind)."""
    return {
        "trellis": torch.stack([m.trellis for m in mats]),
        "suh": torch.stack([m.suh for m in mats]),
        "svh": torch.stack([m.svh for m in mats]),
    }
