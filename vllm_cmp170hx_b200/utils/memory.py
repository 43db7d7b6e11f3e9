"""Memory attribution and the KV / state plan line.

``attribute(model)`` sums the resident bytes of parameters and buffers by
module group (embedding, attention, routed experts, shared experts, dense MLP,
norms, LM head); ``kv_plan(runner)`` describes the paged latent cache, the
indexer key cache and the recurrent-state slots.  Both are logged once after
load when ``VLLM_B200_MEM_ATTRIBUTION`` / ``VLLM_B200_KV_PLAN_LOG`` are set
(the reference's ``VLLM_MEM_ATTRIBUTION``, vllm_sm80/worker/mem_attribution.py:62-276,
and ``VLLM_KV_PLAN_LOG``, vllm_sm80/envs.py:584).
"""

from __future__ import annotations

import collections
import logging

import torch

log = logging.getLogger("vllm_cmp170hx_b200")


def _tensor_bytes(obj) -> int:
    n = 0
    for v in vars(obj).values() if hasattr(obj, "__dict__") else []:
        if isinstance(v, torch.Tensor):
            n += v.numel() * v.element_size()
    return n


def group_of(name: str) -> str:
    if name.startswith("embed"):
        return "embedding"
    if name.startswith("lm_head"):
        return "lm_head"
    if ".attn." in name:
        return "attention"
    if ".mlp.experts" in name:
        return "routed_experts"
    if ".mlp.shared" in name:
        return "shared_experts"
    if ".mlp." in name:
        return "mlp"
    if "norm" in name:
        return "norms"
    return "other"


def attribute(model: torch.nn.Module) -> dict[str, int]:
    out: dict[str, int] = collections.defaultdict(int)
    seen = set()
    for name, p in list(model.named_parameters()) + list(model.named_buffers()):
        if p.data_ptr() in seen:
            continue
        seen.add(p.data_ptr())
        out[group_of(name)] += p.numel() * p.element_size()
    # expert containers are plain dataclasses holding tensors (not parameters)
    for name, mod in model.named_modules():
        ex = getattr(mod, "experts", None)
        if ex is not None and not isinstance(ex, torch.nn.Module):
            out["routed_experts"] += _tensor_bytes(ex)
    return dict(out)


def kv_plan(runner) -> dict:
    lat = sum(t.numel() * t.element_size() for c in runner.mla_caches.values() for t in c)
    st = sum(t.numel() * t.element_size() for c in runner.kda_states.values() for t in c)
    return {"blocks": runner.num_blocks, "block_size": runner.block_size, "mla_layers": len(runner.mla_caches),
            "kda_layers": len(runner.kda_states), "state_slots": getattr(runner, "num_slots", 0),
            "latent_cache_bytes": lat, "state_bytes": st,
            "tokens_capacity": runner.num_blocks * runner.block_size}


def log_attribution(model, rank: int = 0) -> dict[str, int]:
    a = attribute(model)
    total = sum(a.values())
    log.info("memory attribution rank %d: %s (total %.2f GiB)", rank,
             ", ".join(f"{k} {v / 2**30:.2f} GiB" for k, v in sorted(a.items(), key=lambda kv: -kv[1])), total / 2**30)
    return a


def log_kv_plan(runner, rank: int = 0) -> dict:
    p = kv_plan(runner)
    log.info("KV plan rank %d: %s", rank, p)
    return p
