"""Profiler trace helpers: an execution trace beside each kineto trace, and serial trace export.

* ``execution_trace(stem)``: a ``torch.profiler.ExecutionTraceObserver`` runs for
  the lifetime of the block and writes ``<stem>.et.json`` next to the
  profiler's own trace (the reference's ``VLLM_SM80_EXECUTION_TRACE``,
  vllm_sm80/worker/execution_trace.py:1-20).
* ``serial_export(prof, path, rank, world, marker_dir)``: ranks write their
  traces one after another in rank order, each waiting for the previous
  rank's marker file, so N ranks never serialize N traces into host memory at
  once (``VLLM_SM80_SERIAL_TRACE_EXPORT``, vllm_sm80/worker/trace_export.py:1-20).
"""

from __future__ import annotations

import contextlib
import os
import time

import torch


@contextlib.contextmanager
def execution_trace(stem: str):
    et = torch.profiler.ExecutionTraceObserver()
    et.register_callback(stem + ".et.json")
    et.start()
    try:
        yield et
    finally:
        et.stop()
        et.unregister_callback()


def marker_path(marker_dir: str, rank: int) -> str:
    return os.path.join(marker_dir, f"trace_export.rank{rank}.done")


def serial_export(prof, path: str, rank: int, world: int, marker_dir: str, timeout_s: float = 600.0,
                  poll_s: float = 0.05) -> str:
    """Export `prof`'s chrome trace to `path` after rank - 1 finished its own export."""
    os.makedirs(marker_dir, exist_ok=True)
    if rank > 0:
        prev = marker_path(marker_dir, rank - 1)
        t0 = time.monotonic()
        while not os.path.exists(prev):
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"rank {rank - 1} did not finish its trace export")
            time.sleep(poll_s)
    prof.export_chrome_trace(path)
    with open(marker_path(marker_dir, rank), "w") as f:
        f.write(path)
    return path


def clear_markers(marker_dir: str, world: int) -> None:
    for r in range(world):
        try:
            os.remove(marker_path(marker_dir, r))
        except FileNotFoundError:
            pass
