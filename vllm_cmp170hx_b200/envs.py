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
_declare("VLLM_B200_ALLREDUCE", str, "symm", "TP all-reduce transport: 'symm' (own NVLink peer-memory kernels, "
         "read by parallel/symm.py) or 'nccl'")
_declare("VLLM_B200_ALLREDUCE_MAX_BYTES", int, 0, "largest message the symmetric-memory all-reduce takes (0: the "
         "tuning table's allreduce/symm_max_bytes)")
_declare("VLLM_B200_ALLREDUCE_WAIT_S", float, 10.0, "bounded wait of the peer-memory kernels before they report")
_declare("VLLM_B200_FUSED_GEMM_AR", _bool, True, "row-parallel GEMM and MoE combine fused with the all-reduce "
         "(replicated-token layout)")
_declare("VLLM_B200_EP_DISPATCH", str, "symm", "expert-parallel steps: 'symm' (sequence-parallel layout on the fused "
         "peer-store kernels), 'nccl' (the same layout on torch.distributed) or 'off' (replicated tokens)")
# --- kernels ------------------------------------------------------------------------------------
_declare("VLLM_B200_CUDA_GRAPHS", _bool, True, "capture decode steps in CUDA graphs (0: every step eager)")
_declare("VLLM_B200_GEMM_SPLITK", int, 0, "force the split-K factor of the bf16 GEMM (0 = shape-chosen)")
_declare("VLLM_B200_EXL3_TILE_ROWS", int, 0, "rows per EXL3 expert work item, 16 / 32 / 64 / 128 (0 = batch-chosen)")
_declare("VLLM_B200_EXL3_DECODERS", str, "", "decoder warps of the EXL3 GEMM: '8' or '16' for both passes, or "
         "'G,D' for the gate/up and the down pass ('' = the build's default; read by csrc/exl3.cu)")
_declare("VLLM_B200_KDA_PREFILL", str, "chunked", "KDA prefill: 'chunked' (sequences of >= 64 tokens in chunks of 64 "
         "on the tensor cores, read by ops/kda.py) or 'recurrent' (token by token)")
_declare("VLLM_B200_SPARSE_MLA_SPLITS", int, 0, "position splits of the sparse-MLA attention (0 = auto)")
_declare("VLLM_B200_SHARED_EXPERT_STREAM", _bool, False, "MoE layers run the shared expert on a second CUDA stream "
         "beside the routed experts' assignment and rotation, joined before the combine (read by models/hybrid.py)")
_declare("VLLM_B200_PP_SPLIT_DRAFTS", _bool, False, "pipeline parallel speculative decoding: the drafts reach the "
         "other stages by an asynchronous broadcast waited for right before the first stage's forward, the draft "
         "counts (known on every stage) schedule the step meanwhile (read by engine/runner.py)")
_declare("VLLM_B200_PP_DRAFT_TAIL_STAGE", int, -1, "pipeline parallel DFlash drafting: the stage (below the last) "
         "that computes the drafter's tail -- the lm_head over the block's hidden states and the greedy picks -- and "
         "roots the drafts' broadcast; -1 keeps it on the last stage (read by engine/runner.py)")
_declare("VLLM_B200_MLA_DP", _bool, True, "with expert parallelism, sparse-MLA layers hold all heads and attend "
         "data-parallel (each rank its own tokens) in the sequence-parallel layout")
# --- scheduling ---------------------------------------------------------------------------------
_declare("VLLM_B200_FAIR_PREFILL_SHORT_BYPASS", int, 0, "prompts up to this length skip the partial-prefill cap")
_declare("VLLM_B200_ADAPTIVE_K", str, "", "adaptive draft count policy ('' off, 'by_load', 'accept')")
_declare("VLLM_B200_ADAPTIVE_DEPTH", str, "", "per-request verify depth policy file (dspark-depth-policy/1)")
_declare("VLLM_B200_DEPTH_HINT", str, "", "verify width per step from the requests' last rounds: 'full=W,..;base=W,..' "
         "indexed by the requests held (read by engine/llm_engine.py)")
_declare("VLLM_B200_OVERRIDE", str, "", "override sidecar manifest restoring plain tensors at source precision")
_declare("VLLM_B200_NO_PDL", bool, False, "launch kernels without programmatic dependent launch (profiling: each kernel charged its own time)")
_declare("VLLM_B200_OVERRIDE_SHA256", str, "", "pinned sha256 of the override manifest")
# --- serving --------------------------------------------------------------------------------------
_declare("VLLM_B200_TOOL_CHOICE_NONE_MASK", _bool, False, "with tool_choice='none', parsers that have one (glm45, "
         "glm47, ling3) ban their tool-call opener token at decode time (read by api/parsers.py)")
# --- storage-backed embeddings ------------------------------------------------------------------
_declare("VLLM_B200_PLE_READ_RETRIES", int, 3, "retries of a failed PLE/Engram row read (1 ms doubling backoff)")
_declare("VLLM_B200_ROW_CACHE_GIB", float, 0.0, "host LRU cache of table rows read from storage (0 = the table's "
         "own row count)")
# --- diagnostics --------------------------------------------------------------------------------
_declare("VLLM_B200_LIGHT_TIMING", str, "", "device-timed per-scope profiler (JSON spec or '1')")
_declare("VLLM_B200_EXECUTION_TRACE", _bool, False, "record a torch execution trace beside profiler traces")
_declare("VLLM_B200_SERIAL_TRACE_EXPORT", _bool, False, "ranks write profiler traces one after another")
_declare("VLLM_B200_CAPTURE", str, "", "TOML spec of kernel calls to save with inputs/outputs")
_declare("VLLM_B200_MEM_ATTRIBUTION", _bool, False, "log resident bytes per module group after load")
_declare("VLLM_B200_STATE_INDEX_CHECK", _bool, False, "range-check state/cache indices on the host before launch")
_declare("VLLM_B200_KV_PLAN_LOG", _bool, False, "log the KV/state memory plan")
_declare("VLLM_B200_TUNING_FILE", str, "", "per-card tuning table to use instead of the device's own")
_declare("VLLM_B200_DEV_AB_SWITCH", str, "", "dev: capture both arms of a switch and flip between steps")
_declare("VLLM_B200_HOT_SWAP", str, "", "dev: swap implementation pairs between steps")

# reference name -> equivalent here
ALIASES = {
    "VLLM_SM80_ALLREDUCE": "VLLM_B200_ALLREDUCE",
    "VLLM_DSPARK_ADAPTIVE_DEPTH": "VLLM_B200_ADAPTIVE_DEPTH",
    "VLLM_DSPARK_DEPTH_HINT": "VLLM_B200_DEPTH_HINT",
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
    "VLLM_FAIR_PREFILL_SHORT_BYPASS": "VLLM_B200_FAIR_PREFILL_SHORT_BYPASS",
    "VLLM_DEV_AB_SWITCH": "VLLM_B200_DEV_AB_SWITCH",
    "VLLM_HOT_SWAP": "VLLM_B200_HOT_SWAP",
    "VLLM_TOOL_CHOICE_NONE_MASK": "VLLM_B200_TOOL_CHOICE_NONE_MASK",
    "VLLM_EXL3_PLE_READ_RETRIES": "VLLM_B200_PLE_READ_RETRIES",
    "VLLM_PP_SPLIT_DRAFT_EVENT": "VLLM_B200_PP_SPLIT_DRAFTS",
    "VLLM_PP_DRAFT_TAIL_STAGE": "VLLM_B200_PP_DRAFT_TAIL_STAGE",
}

# reference switches whose behaviour is always on here (no switch): accepted, warned about
ALWAYS_ON = {
    "VLLM_SM80_SHARD_ARGMAX": "greedy sampling always combines per-vocab-shard winners (no logits gather)",
    "VLLM_PP_PACKED_HOP": "pipeline boundary tensors always travel as one packed message",
    "VLLM_PP_HOP_NO_METADATA": "pipeline hops never send per-hop metadata (shapes follow from the step)",
    "VLLM_SM80_TOPK_CANONICAL_TIES": "the indexer top-k always breaks ties by the lowest position",
    "VLLM_MOE_DETERMINISTIC_ALIGN": "the expert assignment is always a deterministic counting sort",
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
        elif k in ALWAYS_ON:
            msgs.append(f"{k} has no effect here: {ALWAYS_ON[k]}")
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
