"""Dev A/B switching and hot swaps without a restart (development only).

* A **switch** has two arms, each a function that puts the engine in one
  configuration; ``DevAB.flip()`` moves to the other arm between steps (never
  inside one).  Built-in switches: ``collectives`` (fused symmetric-memory
  kernels / NCCL baseline), ``cuda_graphs`` (decode graphs / eager),
  ``attention_splits`` (automatic position splits / one split).  Selected with
  ``VLLM_B200_DEV_AB_SWITCH=<switch>``; in a multi-rank server the flip rides on
  rank 0's per-step control message so every rank flips at the same step.
* A **hot swap** replaces an entry point with an alternative implementation
  (``VLLM_B200_HOT_SWAP=<pair>[,<pair>]``), e.g. ``gemm:torch`` runs the dense
  projections on ``torch.matmul`` to compare a kernel against the library.

The reference captures graphs for both arms and switches while drained
(vllm_sm80/dev_ab.py:1-40, ``SWITCHES`` :918) and swaps pairs between steps
(vllm_sm80/hot_swap.py:100 ``HotPair``, :279 ``HOT_PAIRS``).
"""

from __future__ import annotations

import importlib
import logging
from dataclasses import dataclass
from typing import Callable

import torch

from .. import envs

log = logging.getLogger("vllm_cmp170hx_b200")


@dataclass
class Switch:
    name: str
    arm_a: Callable
    arm_b: Callable
    doc: str


def _collectives(on: bool):
    def apply(engine):
        from ..parallel import comm, symm

        if on:
            if getattr(engine, "_ab_fused", None) is not None:
                comm.enable_fused(*engine._ab_fused)
            elif pstate_tp(engine) > 1:
                symm.enable_for_engine(engine)
        else:
            engine._ab_fused = (comm._FUSED["symm"], comm._FUSED["fused"])
            comm.enable_fused(None, None)
    return apply


def pstate_tp(engine) -> int:
    from ..parallel import state as pstate

    return pstate.get().tp_size


def _graphs(on: bool):
    def apply(engine):
        engine.runner.cfg.enforce_eager = not on
    return apply


def _splits(auto: bool):
    def apply(engine):
        from ..ops import mla

        if auto:
            if hasattr(mla, "_ab_pick"):
                mla.pick_splits = mla._ab_pick
        else:
            mla._ab_pick = getattr(mla, "_ab_pick", mla.pick_splits)
            mla.pick_splits = lambda *a, **k: 1
    return apply


SWITCHES: dict[str, Switch] = {
    "collectives": Switch("collectives", _collectives(True), _collectives(False),
                          "fused symmetric-memory collectives / NCCL baseline"),
    "cuda_graphs": Switch("cuda_graphs", _graphs(True), _graphs(False), "decode CUDA graphs / eager"),
    "attention_splits": Switch("attention_splits", _splits(True), _splits(False),
                               "automatic sparse-attention splits / one split"),
}


class DevAB:
    def __init__(self, engine, switch: str):
        if switch not in SWITCHES:
            raise KeyError(f"unknown A/B switch {switch!r}; known: {sorted(SWITCHES)}")
        self.engine, self.switch, self.arm = engine, SWITCHES[switch], "a"
        self.switch.arm_a(engine)

    @staticmethod
    def from_env(engine) -> "DevAB | None":
        name = envs.get("VLLM_B200_DEV_AB_SWITCH")
        return DevAB(engine, name) if name else None

    def flip(self) -> str:
        """Move to the other arm (call between steps)."""
        self.arm = "b" if self.arm == "a" else "a"
        (self.switch.arm_b if self.arm == "b" else self.switch.arm_a)(self.engine)
        log.info("A/B switch %s: arm %s", self.switch.name, self.arm)
        return self.arm


# ------------------------------------------------------------------------------------------ hot swaps
def _torch_gemm(x, w, bias=None, out=None, splits=0, out_dtype=torch.bfloat16):
    y = torch.nn.functional.linear(x, w, bias).to(out_dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


HOT_PAIRS: dict[str, tuple[str, str, Callable]] = {
    "gemm:torch": ("vllm_cmp170hx_b200.ops", "gemm", _torch_gemm),
}


class HotSwap:
    def __init__(self, pairs: list[str]):
        self.pairs = pairs
        self.saved: list[tuple] = []

    @staticmethod
    def from_env() -> "HotSwap | None":
        spec = envs.get("VLLM_B200_HOT_SWAP")
        return HotSwap([p.strip() for p in spec.split(",") if p.strip()]) if spec else None

    def swap_in(self) -> None:
        for name in self.pairs:
            modname, attr, fn = HOT_PAIRS[name]
            mod = importlib.import_module(modname)
            self.saved.append((mod, attr, getattr(mod, attr)))
            setattr(mod, attr, fn)

    def swap_out(self) -> None:
        for mod, attr, fn in reversed(self.saved):
            setattr(mod, attr, fn)
        self.saved = []
