"""Platform guard: the CUDA path of this package runs on sm_100 (B200) only.

The reference refuses to start when its plugin or platform is not the one
loaded (vllm_sm80/guard.py:16,42) and probes sm_80 as the last check of
every kernel gate (vllm_sm80/kernels/_platform.py:15).  Here the probe is
for compute capability 10.0 and for the native extension's ABI stamp.
"""

from __future__ import annotations

import functools

import torch

from . import _ext


class UnsupportedPlatform(RuntimeError):
    pass


@functools.cache
def is_sm100(device: int | None = None) -> bool:
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(device) == (10, 0)


def check_platform(device: torch.device | None = None) -> None:
    """Raise unless `device` is a B200-class GPU with the extension built."""
    if device is not None and device.type != "cuda":
        return
    if not torch.cuda.is_available():
        raise UnsupportedPlatform("no CUDA device is visible")
    idx = device.index if device is not None and device.index is not None else torch.cuda.current_device()
    cap = torch.cuda.get_device_capability(idx)
    if cap != (10, 0):
        raise UnsupportedPlatform(f"device {idx} has compute capability {cap}; the kernels are built for sm_100a only")
    _ext.load()
