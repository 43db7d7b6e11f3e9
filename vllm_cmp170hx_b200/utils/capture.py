"""Kernel-call capture: save selected op calls with their inputs and outputs.

A TOML spec (``VLLM_B200_CAPTURE=<file>``) names the ops and limits::

    dir = "captures"            # output directory (one subdirectory per rank)
    ops = ["gemm", "exl3_moe"]  # entry points of vllm_cmp170hx_b200.ops / ops.moe / ops.mla / ops.kda
    max_calls = 4               # per op
    every = 1                   # keep one call in `every`

Each kept call is written as ``<op>.<n>.pt`` (positional and keyword tensor
arguments moved to the host, and the result) and listed in ``index.jsonl``, so
a failing shape can be replayed against the oracle offline.  Captures run on
eager steps; calls inside CUDA-graph capture are skipped (their values would
only exist at replay).  The reference's ``VLLM_SM80_CAPTURE``
(vllm_sm80/capture.py:1-70, ``Record`` :367) saves EXL3, attention and mHC
calls the same way.
"""

from __future__ import annotations

import functools
import json
import os
import tomllib

import torch

from .. import envs

_MODULES = ("vllm_cmp170hx_b200.ops", "vllm_cmp170hx_b200.ops.moe", "vllm_cmp170hx_b200.ops.mla",
            "vllm_cmp170hx_b200.ops.kda", "vllm_cmp170hx_b200.ops.dequant", "vllm_cmp170hx_b200.ops.sampling")


def _host(x):
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", copy=True)
    if isinstance(x, (list, tuple)):
        return type(x)(_host(v) for v in x)
    if isinstance(x, dict):
        return {k: _host(v) for k, v in x.items()}
    return x


class KernelCapture:
    def __init__(self, ops: list[str], out_dir: str, max_calls: int = 4, every: int = 1, rank: int = 0):
        self.ops, self.max_calls, self.every = list(ops), max_calls, max(1, every)
        self.dir = os.path.join(out_dir, f"rank{rank}")
        os.makedirs(self.dir, exist_ok=True)
        self.seen: dict[str, int] = {}
        self.kept: dict[str, int] = {}
        self._restore: list[tuple] = []

    @staticmethod
    def from_env(rank: int = 0) -> "KernelCapture | None":
        path = envs.get("VLLM_B200_CAPTURE")
        if not path:
            return None
        with open(path, "rb") as f:
            spec = tomllib.load(f)
        return KernelCapture(spec.get("ops", []), spec.get("dir", "captures"), int(spec.get("max_calls", 4)),
                             int(spec.get("every", 1)), rank)

    def install(self) -> "KernelCapture":
        import importlib

        for name in self.ops:
            for modname in _MODULES:
                mod = importlib.import_module(modname)
                fn = getattr(mod, name, None)
                if callable(fn) and not getattr(fn, "_b200_capture", False):
                    wrapped = self._wrap(name, fn)
                    setattr(mod, name, wrapped)
                    self._restore.append((mod, name, fn))
        return self

    def uninstall(self) -> None:
        for mod, name, fn in self._restore:
            setattr(mod, name, fn)
        self._restore = []

    def _wrap(self, name, fn):
        @functools.wraps(fn)
        def inner(*args, **kwargs):
            out = fn(*args, **kwargs)
            capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
            n = self.seen.get(name, 0)
            self.seen[name] = n + 1
            if not capturing and n % self.every == 0 and self.kept.get(name, 0) < self.max_calls:
                k = self.kept.get(name, 0)
                self.kept[name] = k + 1
                path = os.path.join(self.dir, f"{name}.{k}.pt")
                torch.save({"op": name, "args": _host(args), "kwargs": _host(kwargs), "out": _host(out)}, path)
                with open(os.path.join(self.dir, "index.jsonl"), "a") as f:
                    shapes = [list(a.shape) for a in args if isinstance(a, torch.Tensor)]
                    f.write(json.dumps({"op": name, "call": n, "file": os.path.basename(path), "shapes": shapes}) + "\n")
            return out

        inner._b200_capture = True
        return inner
