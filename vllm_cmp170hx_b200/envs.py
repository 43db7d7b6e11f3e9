"""Environment variables of the framework: one typed table, read once.

Modelled on the reference's flag table (vllm_sm80/envs.py:1-60,
`register_env_vars` :1705, `RETIRED_ENV_VARS` :1276): every variable is
declared here with a type, a default and a one-line description; reading an
undeclared ``VLLM_B200_*`` name is an error; each feature gate logs once
whether it is active (:func:`log_gate`).

Reference names that have a B200 equivalent are accepted as aliases (with a
warning naming the new variable); sm_80-only names are retired and ignored
with a warning.  Defaults are the product configuration of this build: the
B200 kernels and the fused collectives are on, diagnostics are off.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Any, Callable

log = logging.getLogger("vllm_cmp170hx_b200")


def _bool(v: str) -> bool:
    return v.strip().lower() in ("1", "true", "yes", "on")


@dataclass(frozen=True)
class Var:
    name: str
    type: Callable[[str], Any]
    default: Any
    doc: str


VARS: dict[str, Var] = {}


def _declare(name: str, typ, default, doc: str) -> None:
    assert name not in VARS, name
    VARS[name] = Var(name, typ, default, doc)


# --- collectives --------------------------------------------------------------------------------
_declare("VLLM_B200_ALLREDUCE", str, "symm", "TP all-reduce transport: 'symm' (own NVLink peer-memory kernel) or 'nccl'")
_declare("VLLM_B200_ALLREDUCE_MAX_BYTES", int, 16 << 20, "largest message the symmetric-memory all-reduce takes")
_declare("VLLM_B200_ALLREDUCE_WAIT_S", float, 10.0, "bounded wait of the peer-memory kernels before they report")
_declare("VLLM_B200_FUSED_GEMM_AR", _bool, True, "row-parallel GEMM fused with the all-reduce (tile push)")
_declare("VLLM_B200_EP_DISPATCH", str, "symm", "expert-parallel dispatch/combine: 'symm' or 'nccl'")
_declare("VLLM_B200_PP_PACKED_HOP", _bool, True, "pipeline boundary tensors packed into one send/recv")
_declare("VLLM_B200_PP_HOP_NO_METADATA", _bool, False, "skip the per-hop metadata message after the handshake")
# --- kernels ------------------------------------------------------------------------------------
_declare("VLLM_B200_CUDA_GRAPHS", _bool, True, "capture decode steps in CUDA graphs")
_declare("VLLM_B200_GEMM_SPLITK", int, 0, "force the split-K factor of the bf16 GEMM (0 = shape-chosen)")
_declare("VLLM_B200_EXL3_TILE_ROWS", int, 0, "rows per EXL3 expert work item (0 = batch-chosen)")
_declare("VLLM_B200_SPARSE_MLA_SPLITS", int, 0, "position splits of the sparse-MLA attention (0 = auto)")
_declare("VLLM_B200_KDA_PREFILL", str, "recurrent", "KDA prefill kernel: 'recurrent' (token loop) or 'chunked'")
_declare("VLLM_B200_SHARD_ARGMAX", _bool, True, "greedy sampling by per-shard winners (no logits gather)")
_declare("VLLM_B200_TOPK_CANONICAL_TIES", _bool, True, "indexer top-k: lowest position wins ties")
_declare("VLLM_B200_MOE_DETERMINISTIC_ALIGN", _bool, True, "counting-sort expert assignment (deterministic)")
# --- scheduling ---------------------------------------------------------------------------------
_declare("VLLM_B200_FAIR_PREFILL_SHORT_BYPASS", int, 0, "prompts up to this length skip the partial-prefill cap")
_declare("VLLM_B200_ADAPTIVE_K", str, "", "adaptive draft count policy ('' off, 'by_load', 'accept')")
_declare("VLLM_B200_ADAPTIVE_DEPTH", str, "", "per-request verify depth policy file (dspark-depth-policy/1)")
_declare("VLLM_B200_OVERRIDE", str, "", "override sidecar manifest restoring plain tensors at source precision")
_declare("VLLM_B200_NO_PDL", bool, False, "launch kernels without programmatic dependent launch (profiling: each kernel charged its own time)")
_declare("VLLM_B200_OVERRIDE_SHA256", str, "", "pinned sha256 of the override manifest")
# --- storage-backed embeddings ------------------------------------------------------------------
_declare("VLLM_B200_PLE_READ_RETRIES", int, 3, "retries of a failed PLE/Engram row read (1 ms doubling backoff)")
_declare("VLLM_B200_ROW_CACHE_GIB", float, 0.0, "host LRU cache of table rows read from storage")
# --- diagnostics --------------------------------------------------------------------------------
_declare("VLLM_B200_LIGHT_TIMING", str, "", "device-timed per-scope profiler (JSON spec or '1')")
_declare("VLLM_B200_EXECUTION_TRACE", _bool, False, "record a torch execution trace beside profiler traces")
_declare("VLLM_B200_SERIAL_TRACE_EXPORT", _bool, False, "ranks write profiler traces one after another")
_declare("VLLM_B200_CAPTURE", str, "", "TOML spec of kernel calls to save with inputs/outputs")
_declare("VLLM_B200_MEM_ATTRIBUTION", _bool, False, "log resident bytes per module group after load")
_declare("VLLM_B200_STATE_INDEX_CHECK", _bool, False, "range-check state/cache indices on the host before launch")
_declare("VLLM_B200_KV_PLAN_LOG", _bool, False, "log the KV/state memory plan")
_declare("VLLM_B200_TUNING_FILE", str, "", "per-card tuning table to use instead of the device's own")
_declare("VLLM_B200_TOOL_CHOICE_NONE_MASK", _bool, False, "mask tool-call start tokens when tool_choice='none'")
_declare("VLLM_B200_DEV_AB_SWITCH", str, "", "dev: capture both arms of a switch and flip between steps")
_declare("VLLM_B200_HOT_SWAP", str, "", "dev: swap implementation pairs between steps")

# reference name -> equivalent here
ALIASES = {
    "VLLM_SM80_ALLREDUCE": "VLLM_B200_ALLREDUCE",
    "VLLM_DSPARK_ADAPTIVE_DEPTH": "VLLM_B200_ADAPTIVE_DEPTH",
    "VLLM_EXL3_OVERRIDE": "VLLM_B200_OVERRIDE",
    "VLLM_EXL3_OVERRIDE_SHA256": "VLLM_B200_OVERRIDE_SHA256",
    "VLLM_SM80_LIGHT_TIMING": "VLLM_B200_LIGHT_TIMING",
    "VLLM_SM80_EXECUTION_TRACE": "VLLM_B200_EXECUTION_TRACE",
    "VLLM_SM80_SERIAL_TRACE_EXPORT": "VLLM_B200_SERIAL_TRACE_EXPORT",
    "VLLM_SM80_CAPTURE": "VLLM_B200_CAPTURE",
    "VLLM_MEM_ATTRIBUTION": "VLLM_B200_MEM_ATTRIBUTION",
    "VLLM_STATE_INDEX_CHECK": "VLLM_B200_STATE_INDEX_CHECK",
    "VLLM_KV_PLAN_LOG": "VLLM_B200_KV_PLAN_LOG",
    "VLLM_SM80_TUNING_FILE": "VLLM_B200_TUNING_FILE",
    "VLLM_SM80_SHARD_ARGMAX": "VLLM_B200_SHARD_ARGMAX",
    "VLLM_FAIR_PREFILL_SHORT_BYPASS": "VLLM_B200_FAIR_PREFILL_SHORT_BYPASS",
    "VLLM_PP_PACKED_HOP": "VLLM_B200_PP_PACKED_HOP",
    "VLLM_PP_HOP_NO_METADATA": "VLLM_B200_PP_HOP_NO_METADATA",
    "VLLM_TOOL_CHOICE_NONE_MASK": "VLLM_B200_TOOL_CHOICE_NONE_MASK",
    "VLLM_DEV_AB_SWITCH": "VLLM_B200_DEV_AB_SWITCH",
    "VLLM_HOT_SWAP": "VLLM_B200_HOT_SWAP",
    "VLLM_EXL3_PLE_READ_RETRIES": "VLLM_B200_PLE_READ_RETRIES",
    "VLLM_SM80_TOPK_CANONICAL_TIES": "VLLM_B200_TOPK_CANONICAL_TIES",
    "VLLM_MOE_DETERMINISTIC_ALIGN": "VLLM_B200_MOE_DETERMINISTIC_ALIGN",
}

# reference switches of sm_80-only code paths: accepted, ignored, warned about
RETIRED_PREFIXES = ("VLLM_AMPERE_", "VLLM_FLA_", "VLLM_GLM5_THIN_GEMM", "VLLM_THIN_GEMM", "VLLM_SM80_KDA_PREFILL",
                    "VLLM_HOST_ALLREDUCE", "VLLM_GLM5_HOST_ALLREDUCE", "VLLM_CUSTOM_ALLREDUCE_FLAGS",
                    "VLLM_CUSTOM_ALLREDUCE_PCIE_P2P", "VLLM_ALLOW_PCIE_P2P_CUSTOM_ALLREDUCE")

_warned: set[str] = set()
_cache: dict[str, Any] = {}


def _warn_once(key: str, msg: str) -> None:
    if key not in _warned:
        _warned.add(key)
        log.warning(msg)


def get(name: str) -> Any:
    if name not in VARS:
        raise KeyError(f"undeclared environment variable {name}")
    if name in _cache:
        return _cache[name]
    var = VARS[name]
    raw = os.environ.get(name)
    if raw is None:
        for old, new in ALIASES.items():
            if new == name and old in os.environ:
                _warn_once(old, f"{old} is the reference's name; use {name}")
                raw = os.environ[old]
                break
    if raw is None or (raw == "" and var.type is not str):
        val = var.default
    else:
        val = var.type(raw)
    _cache[name] = val
    return val


def reset_cache() -> None:
    _cache.clear()


def check_environment() -> list[str]:
    """Warn about retired reference switches and unknown VLLM_B200_* names; returns the warnings."""
    msgs = []
    for k in os.environ:
        if k.startswith("VLLM_B200_") and k not in VARS:
            msgs.append(f"unknown variable {k} (not declared in vllm_cmp170hx_b200.envs)")
        elif any(k.startswith(p) for p in RETIRED_PREFIXES):
            msgs.append(f"{k} switches an sm_80-only code path of the reference; it has no effect here")
    for m in msgs:
        _warn_once(m, m)
    return msgs


def log_gate(feature: str, active: bool, why: str = "") -> None:
    """One startup line per gated feature: active, or why the gate is closed."""
    key = f"gate:{feature}"
    if key in _warned:
        return
    _warned.add(key)
    log.info("%s: %s%s", feature, "active" if active else "off", f" ({why})" if why else "")


def describe() -> str:
    return "\n".join(f"{v.name} [{v.type.__name__ if hasattr(v.type, '__name__') else v.type}] "
                     f"default={v.default!r}: {v.doc}" for v in VARS.values())
