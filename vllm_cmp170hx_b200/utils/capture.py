"""Kernel-call capture: save selected op calls with their inputs and outputs.

A TOML spec (``VLLM_B200_CAPTURE=<file>``) names the ops and limits::

    dir = "captures"            # output directory (one subdirectory per rank)
    ops = ["gemm", "exl3_moe"]  # entry points of vllm_cmp170hx_b200.ops / ops.moe / ops.mla / ops.kda
    max_calls = 4               # per op
    every = 1                   # keep one call in `every`

Each kept call is written as ``<op>.<n>.pt`` (positional and keyword tensor
arguments as they were before the call, moved to the host, and the result) and
listed in ``index.jsonl``, so a failing shape can be replayed against the
oracle offline: :func:`replay` re-runs one saved call on a device of choice
(CPU tensors take the fp32 oracle path of every op) and compares the result
with the saved one::

    python -m vllm_cmp170hx_b200.utils.capture replay captures/rank0 --device cpu --tol 0.05  Captures run on
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
            capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
            n = self.seen.get(name, 0)
            self.seen[name] = n + 1
            keep = not capturing and n % self.every == 0 and self.kept.get(name, 0) < self.max_calls
            # the inputs as the op sees them (ops that write into an argument change it)
            saved = (_host(args), _host(kwargs)) if keep else None
            out = fn(*args, **kwargs)
            if keep:
                k = self.kept.get(name, 0)
                self.kept[name] = k + 1
                path = os.path.join(self.dir, f"{name}.{k}.pt")
                torch.save({"op": name, "args": saved[0], "kwargs": saved[1], "out": _host(out)}, path)
                with open(os.path.join(self.dir, "index.jsonl"), "a") as f:
                    shapes = [list(a.shape) for a in args if isinstance(a, torch.Tensor)]
                    f.write(json.dumps({"op": name, "call": n, "file": os.path.basename(path), "shapes": shapes}) + "\n")
            return out

        inner._b200_capture = True
        return inner


def _to(x, device):
    if isinstance(x, torch.Tensor):
        return x.to(device)
    if isinstance(x, (list, tuple)):
        return type(x)(_to(v, device) for v in x)
    if isinstance(x, dict):
        return {k: _to(v, device) for k, v in x.items()}
    return x


def _find_op(name: str):
    import importlib

    for modname in reversed(_MODULES):  # the most specific module first
        fn = getattr(importlib.import_module(modname), name, None)
        if callable(fn):
            return getattr(fn, "__wrapped__", fn)
    raise KeyError(f"no op {name!r} in {_MODULES}")


def _leaves(x):
    if isinstance(x, torch.Tensor):
        return [x]
    if isinstance(x, (list, tuple)):
        return [t for v in x for t in _leaves(v)]
    return []


def replay(path: str, device: str = "cpu") -> float:
    """Re-run one saved call on `device` and return the largest relative difference (max |a - b| / max |b|)
    between its result tensors and the saved ones."""
    rec = torch.load(path, weights_only=False)
    fn = _find_op(rec["op"])
    out = fn(*_to(rec["args"], device), **_to(rec["kwargs"], device))
    worst = 0.0
    for a, b in zip(_leaves(out), _leaves(rec["out"])):
        if a.shape != b.shape:
            return float("inf")
        if not a.is_floating_point():
            worst = max(worst, 0.0 if torch.equal(a.cpu(), b) else float("inf"))
            continue
        d = (a.detach().float().cpu() - b.float()).abs().max().item() if a.numel() else 0.0
        worst = max(worst, d / max(b.float().abs().max().item(), 1e-6) if b.numel() else 0.0)
    return worst


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="replay saved kernel calls")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("replay")
    r.add_argument("dir")
    r.add_argument("--device", default="cpu")
    r.add_argument("--tol", type=float, default=0.05)
    a = ap.parse_args(argv)
    bad = 0
    with open(os.path.join(a.dir, "index.jsonl")) as f:
        for line in f:
            e = json.loads(line)
            d = replay(os.path.join(a.dir, e["file"]), a.device)
            ok = d <= a.tol
            bad += not ok
            print(json.dumps({"file": e["file"], "op": e["op"], "shapes": e["shapes"], "rel_diff": d, "ok": ok}))
    return 1 if bad else 0


if __name__ == "__main__":
    import sys

    sys.exit(main())
