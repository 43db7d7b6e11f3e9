"""Model registry: architecture names of checkpoints -> model classes.

The reference overrides upstream model classes by architecture name
(vllm_sm80/plugin.py:24-51 MODEL_OVERRIDES) and injects HF-config defaults
(:83 HF_CONFIG_DEFAULTS, model_registry.py:72).  Here every supported
architecture maps to one of this package's model classes; configs are read
with :func:`vllm_cmp170hx_b200.config.from_hf_config`.
"""

from __future__ import annotations

import json
from pathlib import Path

from .config import ModelConfig, PRESETS, from_hf_config

ARCHITECTURES = {
    # hybrid KDA / sparse-MLA MoE family (GLM-5.x)
    "Glm5NextForConditionalGeneration": "hybrid",
    "Glm5NextForCausalLM": "hybrid",
    "HybridKdaMlaMoeForCausalLM": "hybrid",
    # DeepSeek-style sparse-MLA MoE (all layers MLA)
    "DeepseekV3ForCausalLM": "hybrid",
    "DeepseekV32ForCausalLM": "hybrid",
    "DeepseekV41ForCausalLM": "hybrid",
    # Qwen3-Next-style linear / full hybrid (the reference's Qwen4Exp classes, sm80_model.py:72-121)
    "Qwen3NextForCausalLM": "hybrid",
    "Qwen4ExpForCausalLM": "hybrid",
    "Qwen4ExpForConditionalGeneration": "hybrid",
}

HF_CONFIG_DEFAULTS = {
    # the DeepSeek-V4.1 head runs in fp32 in the reference (plugin.py:83)
    "DeepseekV41ForCausalLM": {"head_dtype": "float32"},
}


def model_class(kind: str):
    if kind == "hybrid":
        from .models.hybrid import HybridForCausalLM

        return HybridForCausalLM
    raise KeyError(kind)


def resolve(model: str) -> tuple[ModelConfig, str | None]:
    """`model` is a preset name (config3, config4, tiny, ...) or a checkpoint
    directory with config.json.  Returns (config, checkpoint dir or None)."""
    if model in PRESETS:
        return PRESETS[model](), None
    p = Path(model)
    cfg_path = p / "config.json" if p.is_dir() else p
    hf = json.loads(cfg_path.read_text())
    arch = (hf.get("architectures") or ["HybridKdaMlaMoeForCausalLM"])[0]
    if arch not in ARCHITECTURES:
        raise ValueError(f"unsupported architecture {arch}; supported: {sorted(ARCHITECTURES)}")
    hf = {**HF_CONFIG_DEFAULTS.get(arch, {}), **hf}
    return from_hf_config(hf), str(p) if p.is_dir() else None
