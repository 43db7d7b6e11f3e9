"""Dev A/B switching and hot swaps without a restart (development only).

* A **switch** has two arms, each a function that puts the engine in one
  configuration; ``DevAB.flip()`` moves to the other arm between steps (never
  inside one).  Built-in switches (``SWITCHES``): collectives (fused / NCCL),
  CUDA graphs, attention splits, asynchronous scheduling, the shared-expert
  stream, KDA prefill form, EXL3 work-item rows, GEMM split-K, router logits
  precision, prefix caching and the fair-prefill budget; arms that change what
  a decode graph launches drop the captured graphs (captured again on demand).  Selected with
  ``VLLM_B200_DEV_AB_SWITCH=<switch>``; in a multi-rank server the flip rides on
  rank 0's per-step control message so every rank flips at the same step.
* A **hot swap** replaces an entry point with an alternative implementation
  (``VLLM_B200_HOT_SWAP=<pair>[,<pair>]``), e.g. ``gemm:torch`` runs the dense
  projections on ``torch.matmul`` to compare a kernel against the library
  (also ``rms_norm:torch``, ``silu_mul:torch``, ``moe_topk:oracle``).

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


def _env(name: str, value: str | None, recapture: bool):
    """Arm that sets (or clears) an environment switch; arms that change what a decode graph launches drop
    the captured graphs, which are captured again on the next step that needs them."""
    def apply(engine):
        import os

        if value is None:
            os.environ.pop(name, None)
        else:
            os.environ[name] = value
        envs.reset_cache()
        if recapture:
            engine.runner.release_graphs()
    return apply


def _attr(getter, field: str, value, recapture: bool = False):
    """Arm that sets an attribute of a part of the engine (getter(engine) -> object or list of them)."""
    def apply(engine):
        objs = getter(engine)
        for o in objs if isinstance(objs, list) else [objs]:
            setattr(o, field, value)
        if recapture:
            engine.runner.release_graphs()
    return apply


def _moe_layers(engine):
    from ..models.hybrid import MoE

    return [m for m in engine.runner.model.modules() if isinstance(m, MoE)]


def _env_switch(name: str, var: str, a: str | None, b: str, doc: str, recapture: bool = True) -> Switch:
    return Switch(name, _env(var, a, recapture), _env(var, b, recapture), doc)


SWITCHES: dict[str, Switch] = {
    "collectives": Switch("collectives", _collectives(True), _collectives(False),
                          "fused symmetric-memory collectives / NCCL baseline"),
    "cuda_graphs": Switch("cuda_graphs", _graphs(True), _graphs(False), "decode CUDA graphs / eager"),
    "attention_splits": Switch("attention_splits", _splits(True), _splits(False),
                               "automatic sparse-attention splits / one split"),
    "async_scheduling": Switch("async_scheduling", _attr(lambda e: e.cfg.scheduler, "async_scheduling", True),
                               _attr(lambda e: e.cfg.scheduler, "async_scheduling", False),
                               "decode steps scheduled one step ahead / every step read back first"),
    "shared_expert_stream": _env_switch("shared_expert_stream", "VLLM_B200_SHARED_EXPERT_STREAM", "1", "0",
                                        "shared expert on a second stream / inline"),
    "kda_prefill": _env_switch("kda_prefill", "VLLM_B200_KDA_PREFILL", "chunked", "recurrent",
                               "chunked tensor-core KDA prefill / token recurrence", recapture=False),
    "exl3_tile_rows": _env_switch("exl3_tile_rows", "VLLM_B200_EXL3_TILE_ROWS", None, "128",
                                  "batch-chosen EXL3 work-item rows / 128-row items"),
    "gemm_splitk": _env_switch("gemm_splitk", "VLLM_B200_GEMM_SPLITK", None, "1",
                               "shape-chosen GEMM split-K / no split"),
    "router_dtype": Switch("router_dtype", _attr(_moe_layers, "router_out", torch.float32, True),
                           _attr(_moe_layers, "router_out", torch.bfloat16, True),
                           "fp32 router logits / bf16 router logits"),
    "prefix_caching": Switch("prefix_caching", _attr(lambda e: e.scheduler, "prefix_caching", False),
                             _attr(lambda e: e.scheduler, "prefix_caching", True),
                             "no prefix reuse / prefix caching (models without recurrent state)"),
    "fair_prefill": Switch("fair_prefill", _attr(lambda e: e.cfg.scheduler, "prefill_chunk_with_decodes", 0),
                           _attr(lambda e: e.cfg.scheduler, "prefill_chunk_with_decodes", 512),
                           "one step budget / a 512-token prefill-only budget beside the decodes"),
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


def _torch_rms_norm(x, w, eps, out=None):
    xf = x.float()
    y = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _torch_silu_mul(x, limit=0.0, out=None):
    g, u = x.float().chunk(2, -1)
    if limit > 0:
        g, u = g.clamp(max=limit), u.clamp(-limit, limit)
    y = (torch.nn.functional.silu(g) * u).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _torch_topk(logits, k, mode=0, bias=None, scale=1.0, renorm=True):
    from ..oracle import moe as moe_ref

    ids, w = moe_ref.topk(logits.float().cpu(), k, mode, None if bias is None else bias.float().cpu(), scale, renorm)
    return ids.to(logits.device, torch.int32), w.to(logits.device, torch.float32)


HOT_PAIRS: dict[str, tuple[str, str, Callable]] = {
    "gemm:torch": ("vllm_cmp170hx_b200.ops", "gemm", _torch_gemm),
    "rms_norm:torch": ("vllm_cmp170hx_b200.ops", "rms_norm", _torch_rms_norm),
    "silu_mul:torch": ("vllm_cmp170hx_b200.ops", "silu_mul", _torch_silu_mul),
    "moe_topk:oracle": ("vllm_cmp170hx_b200.ops.moe", "topk", _torch_topk),
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
