"""B200-native LLM serving engine (sm_100a kernels, NCCL/NVLink collectives).

Capabilities follow the vllm-sm80 plugin stack (Morrowmake/vllm-cmp170hx):
an OpenAI-compatible server over a continuous-batching engine, hybrid
KDA / sparse-MLA MoE models, EXL3-trellis and Marlin-int4 expert weights,
env-var-gated features that are off by default.  The compute path is
PyTorch plus the hand-written kernels of ``csrc/`` built for sm_100a only.
"""

__version__ = "0.1.0"
