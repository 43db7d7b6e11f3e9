"""Loader of the native `_C` extension.

On a machine with a CUDA device the extension must be present: every op of
``vllm_cmp170hx_b200.ops`` that receives a CUDA tensor runs its sm_100a
kernel and there is no silent eager fallback.  A missing or stale build
raises with the command that builds it.  On a machine without a GPU the
package still imports (CPU tensors take the oracle path of ``oracle/``).
"""

from __future__ import annotations

import functools

import torch

BUILD_HINT = "python setup.py build_ext --inplace   (from the repository root)"
EXPECTED_BUILD_INFO = 100 * 1000 + 3


class ExtensionMissing(RuntimeError):
    pass


@functools.cache
def load():
    """Import `_C` (registers torch.ops.b200.*) and check its ABI stamp."""
    try:
        from . import _C  # noqa: F401
    except ImportError as e:  # pragma: no cover - depends on the build
        raise ExtensionMissing(f"native extension vllm_cmp170hx_b200._C is not built ({e}); run {BUILD_HINT}") from e
    info = int(torch.ops.b200.build_info())
    if info != EXPECTED_BUILD_INFO:
        raise ExtensionMissing(f"stale native extension (build_info {info}, expected {EXPECTED_BUILD_INFO}); "
                               f"run {BUILD_HINT}")
    return _C


def available() -> bool:
    try:
        load()
        return True
    except ExtensionMissing:
        return False


def ops():
    load()
    return torch.ops.b200


@functools.cache
def _status_word(device_index: int) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=f"cuda:{device_index}")


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that bounded device waits OR their error codes into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return _status_word(idx)


ERROR_BITS = {
    1: "mbarrier wait timed out",
    2: "peer flag wait timed out",
    4: "index out of range (access skipped)",
    8: "TMEM allocation did not return",
}


class DeviceStepError(RuntimeError):
    pass


def check_status(device: torch.device, clear: bool = True) -> None:
    """Raise DeviceStepError if a kernel on `device` reported an error (host sync)."""
    raise_status(device, int(status_word(device).item()), clear)


def raise_status(device: torch.device, v: int, clear: bool = True) -> None:
    """Raise DeviceStepError for a status value `v` already read from `device`'s word."""
    if v:
        w = status_word(device)
        if clear:
            w.zero_()
        names = [msg for bit, msg in ERROR_BITS.items() if v & bit]
        raise DeviceStepError(f"device status {v:#x}: {', '.join(names)}")
