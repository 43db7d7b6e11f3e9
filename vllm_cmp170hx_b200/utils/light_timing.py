"""Light timing: a device-timed per-scope profiler that works inside CUDA graphs.

A device ring ``int64[rows, width]`` holds one row per forward pass; column 0
is the row's step number, every other column a named scope edge.  Opening a
row and stamping an edge are single small kernels (``csrc/timing.cu``) that
read ``%globaltimer``; the row index lives in device memory, so stamps that
were captured in a CUDA graph land in the row each replay opens and no host
work happens per step.  ``dump`` writes the ring (``rank<r>.<n>.npz``);
``summarize`` turns a dump into per-scope durations.  The reference's
``VLLM_SM80_LIGHT_TIMING`` profiler works the same way
(vllm_sm80/worker/light_timing.py:1-60, ``LightTimer`` :183).

On CPU tensors the same API records host ``perf_counter_ns`` values (tests).
Enabled by ``VLLM_B200_LIGHT_TIMING`` = ``1`` or a JSON object
``{"rows": 4096, "scopes": "layer" | "block", "dir": "<dump dir>"}``.
"""

from __future__ import annotations

import json
import os
import time

import numpy as np
import torch

from .. import _ext, envs


class LightTimer:
    def __init__(self, device: torch.device, rows: int = 4096, width: int = 512, scopes: str = "layer",
                 out_dir: str = "."):
        self.device = device
        self.rows, self.width = rows, width
        self.scopes = scopes
        self.out_dir = out_dir
        self.cols: dict[str, int] = {}
        self.ring = torch.zeros(rows, width, dtype=torch.int64, device=device)
        self.cursor = torch.full((1,), rows - 1, dtype=torch.int32, device=device)
        self.step = torch.zeros(1, dtype=torch.int64, device=device)
        self.dumps = 0
        self._handles = []

    @staticmethod
    def from_env(device: torch.device) -> "LightTimer | None":
        spec = envs.get("VLLM_B200_LIGHT_TIMING")
        if not spec:
            return None
        cfg = {} if spec.strip() in ("1", "true", "on") else json.loads(spec)
        return LightTimer(device, rows=int(cfg.get("rows", 4096)), width=int(cfg.get("width", 512)),
                          scopes=cfg.get("scopes", "layer"), out_dir=cfg.get("dir", "."))

    # ------------------------------------------------------------------ recording
    def col(self, name: str) -> int:
        c = self.cols.get(name)
        if c is None:
            c = len(self.cols) + 1
            if c >= self.width:
                raise ValueError(f"light timing: more than {self.width - 1} scope edges")
            self.cols[name] = c
        return c

    def open_row(self) -> None:
        if self.device.type == "cuda":
            _ext.ops().timing_open_row(self.ring, self.cursor, self.step)
        else:
            r = (int(self.cursor[0]) + 1) % self.rows
            self.cursor[0] = r
            self.ring[r].zero_()
            self.step += 1
            self.ring[r, 0] = self.step[0]

    def stamp(self, name: str) -> None:
        c = self.col(name)
        if self.device.type == "cuda":
            _ext.ops().timing_stamp(self.ring, self.cursor, c)
        else:
            self.ring[int(self.cursor[0]), c] = time.perf_counter_ns()

    def attach(self, model) -> None:
        """Stamp the edges of every decoder layer (scopes "layer") or of its attention / MLP blocks too
        (scopes "block") through forward hooks, which also run while a graph is captured."""
        for layer in getattr(model, "layers", []):
            name = f"L{layer.idx}"
            self._hook(layer, name)
            if self.scopes == "block":
                self._hook(layer.attn, f"{name}.attn")
                if layer.mlp is not None:
                    self._hook(layer.mlp, f"{name}.mlp")

    def _hook(self, mod, name: str) -> None:
        self._handles.append(mod.register_forward_pre_hook(lambda m, a: self.stamp(name + ">")))
        self._handles.append(mod.register_forward_hook(lambda m, a, o: self.stamp(name + "<")))

    def detach(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles = []

    # ------------------------------------------------------------------ output
    def dump(self, rank: int = 0) -> str:
        os.makedirs(self.out_dir, exist_ok=True)
        path = os.path.join(self.out_dir, f"rank{rank}.{self.dumps}.npz")
        self.dumps += 1
        names = sorted(self.cols, key=self.cols.get)
        np.savez(path, ring=self.ring.cpu().numpy(), names=np.array(names), cols=np.array([self.cols[n] for n in names]))
        return path


def summarize(path: str) -> dict[str, float]:
    """Mean duration (us) of every scope "<name>" between its ">" (enter) and "<" (leave) stamps over
    the recorded rows."""
    d = np.load(path)
    ring, names, cols = d["ring"], list(d["names"]), list(d["cols"])
    rows = ring[ring[:, 0] > 0]
    col = dict(zip(names, cols))
    out = {}
    for n in names:
        if n.endswith(">") and (n[:-1] + "<") in col:
            a, b = rows[:, col[n]], rows[:, col[n[:-1] + "<"]]
            ok = (a > 0) & (b > 0)
            if ok.any():
                out[n[:-1]] = float((b[ok] - a[ok]).mean()) / 1e3
    return out
