"""Canary-guarded output buffers: a race / out-of-bounds detector for kernel outputs.

``Guarded(shape, dtype, device)`` allocates the output with guard rows before and after it (and a guard
tail on every row when ``row_pad`` is given), fills the guards with a canary value -- a NaN bit pattern for
floating point, 0x5A bytes otherwise -- and hands out the inner view; ``check()`` raises ``CanaryError``
naming the first damaged guard element after the kernel ran.  A kernel that writes past its rows, past a
row's end, or into a neighbour's tile of a shared buffer trips it, without compute-sanitizer (the
reference's plan for the same check: canary-padded outputs compared after each launch in tests).
"""

from __future__ import annotations

import torch


class CanaryError(AssertionError):
    pass


def _fill(t: torch.Tensor) -> None:
    if t.is_floating_point():
        t.view(torch.uint8).fill_(0x7F if t.element_size() == 1 else 0xFF)  # an all-ones NaN pattern
    else:
        t.view(torch.uint8).fill_(0x5A)


class Guarded:
    def __init__(self, shape, dtype, device, pad: int = 8, row_pad: int = 0):
        shape = tuple(shape)
        rows = shape[0]
        inner = int(torch.Size(shape[1:]).numel()) if len(shape) > 1 else 1
        self.shape, self.pad, self.row_pad = shape, pad, row_pad
        width = inner + row_pad
        self.buf = torch.empty(pad + rows + pad, width, dtype=dtype, device=device)
        _fill(self.buf)
        self.ref = self.buf.clone()
        body = self.buf[pad:pad + rows].narrow(1, 0, inner)
        # rows with a guard tail keep their stride: the kernel sees [rows, inner] with ld = inner + row_pad
        self.view = body if row_pad else body.view(shape)

    def check(self) -> None:
        rows = self.shape[0]
        inner = self.buf.shape[1] - self.row_pad
        b, r = self.buf.view(torch.uint8), self.ref.view(torch.uint8)
        es = self.buf.element_size()
        regions = [("leading guard rows", b[:self.pad], r[:self.pad]),
                   ("trailing guard rows", b[self.pad + rows:], r[self.pad + rows:])]
        if self.row_pad:
            regions.append(("row guard tails", b[self.pad:self.pad + rows, inner * es:],
                            r[self.pad:self.pad + rows, inner * es:]))
        for name, got, want in regions:
            bad = (got != want).nonzero()
            if bad.numel():
                raise CanaryError(f"{name} written: first damaged byte at {bad[0].tolist()} "
                                  f"({bad.shape[0]} bytes in all)")
