"""Model and engine configuration.

Model configs describe the two model families of the reference's served
models (README.md:32-37 of the reference: GLM-5.3-Flash hybrid KDA/sparse-MLA
MoE, DeepSeek-V4.1-Flash sparse-MLA MoE) in the shapes BASELINE.json names:

* :func:`config3` -- hybrid KDA/MLA MoE: 48 layers at 3:1 KDA:sparse-MLA,
  hidden 2304, 32 heads, 256 routed experts top-8 + 1 shared, expert
  intermediate 1024, EXL3 4-bit (bits_x2 = 8) experts, bf16 dense weights,
  vocab 163840.
* :func:`config4` -- DeepSeek-style sparse-MLA MoE: 43 layers, hidden 4096,
  first 3 layers dense FFN 12288, 256 routed experts top-8 + 1 shared, expert
  intermediate 1536, Marlin int4 group-128 experts, fp8 128x128 block-scaled
  attention weights, 128 heads.
* :func:`config2_layer` -- one sparse-MLA decode layer: 128 heads, kv_lora
  512, qk_nope 128, qk_rope 64, v_head 128, indexer 64 x 128 top-2048.

Engine config mirrors the knobs of the reference's engine settings
(vllm_sm80/config.py:26 `additional_config["sm80"]`, engine_args.py:63
`--prefill-chunk-with-decodes`, `--max-num-partial-prefills`).
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field


@dataclass
class KDAConfig:
    """Linear-attention layers (layer type "kda"): Kimi delta attention (mode "kda": per-channel decay,
    sigmoid output gate) or the gated delta net of Qwen3-Next-style models (mode "gdn": one decay per
    head, SiLU output gate, num_k_heads query / key heads shared by num_heads // num_k_heads value heads)."""
    num_heads: int = 32
    head_dim: int = 128
    conv_kernel: int = 4
    lower_bound: float = -5.0
    mode: str = "kda"
    num_k_heads: int = 0  # gdn: query / key heads (0: num_heads)

    def __post_init__(self):
        if self.mode not in ("kda", "gdn"):
            raise ValueError(f"KDAConfig.mode={self.mode!r}: 'kda' or 'gdn'")
        nk = self.num_k_heads or self.num_heads
        if self.num_heads % nk:
            raise ValueError("KDAConfig: value heads must be a multiple of the query / key heads")


@dataclass
class GQAConfig:
    """Gated grouped-query full attention (layer type "gqa", Qwen3-Next style): per query head
    [q | sigmoid gate], per-head q / k RMSNorm, partial NeoX RoPE, head_dim 256."""
    num_heads: int = 16
    num_kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 10000000.0

    def __post_init__(self):
        if self.head_dim != 256 or self.num_heads % self.num_kv_heads or self.rotary_dim % 2:
            raise ValueError("GQAConfig: head_dim 256, query heads a multiple of key-value heads, even rotary dims")


@dataclass
class MLAConfig:
    num_heads: int = 32
    q_lora_rank: int = 768
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 2048
    rope_theta: float = 10000.0
    rope_interleave: bool = False
    attn_weight_format: str = "bf16"  # or "fp8_block" (128x128 block-scaled e4m3)

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim


@dataclass
class DSAConfig:
    """DeepSeek-V4.1 attention (layer type "dsa"): MQA over 512-wide rows (K = V, RoPE on the last
    64) from a sliding window plus compressed groups chosen by an indexer; per-head sinks; the
    output goes through grouped wo_a then row-parallel wo_b."""
    num_heads: int = 64
    head_dim: int = 512
    rope_dim: int = 64
    q_lora_rank: int = 1536
    window: int = 128
    compress_ratios: list[int] = field(default_factory=list)  # per dsa layer: 0 (window only), 1 or 2
    index_n_heads: int = 32
    index_head_dim: int = 128
    index_topk: int = 512
    index_rank_groups: int = 1  # score rounding groups of the indexer heads (the reference's TP)
    o_groups: int = 8
    o_lora_rank: int = 1024
    rope_theta: float = 10000.0

    def __post_init__(self):
        bad = sorted({r for r in self.compress_ratios if r not in (0, 1, 2)})
        if bad:
            raise ValueError(f"DSAConfig.compress_ratios: ratios {bad} are not supported (0, 1 or 2)")


@dataclass
class MoEConfig:
    num_experts: int = 256
    top_k: int = 8
    intermediate: int = 1024
    num_shared: int = 1
    shared_intermediate: int = 1024
    router: str = "softmax"  # softmax | sigmoid | sqrt_softplus
    routed_scaling: float = 1.0
    renormalize: bool = True
    expert_format: str = "exl3"  # exl3 | marlin | bf16
    exl3_bits_x2: int = 8
    exl3_codebook: int = 2
    swiglu_limit: float = 0.0
    # router logits precision: "float32" (the gate GEMM writes fp32 logits) or "bfloat16" (logits rounded
    # to the model dtype before the top-k), the reference's `moe_router_dtype` switch
    router_dtype: str = "float32"

    def __post_init__(self):
        if self.router_dtype not in ("float32", "bfloat16"):
            raise ValueError(f"MoEConfig.router_dtype={self.router_dtype!r}: 'float32' or 'bfloat16'")

    @property
    def router_mode(self) -> int:
        return {"softmax": 0, "sigmoid": 1, "sqrt_softplus": 2}[self.router]


@dataclass
class ModelConfig:
    name: str = "hybrid-kda-mla-moe"
    vocab_size: int = 163840
    hidden_size: int = 2304
    num_layers: int = 48
    layer_types: list[str] = field(default_factory=list)  # "kda" | "mla" | "dsa" | "gqa" per layer
    mlp_types: list[str] = field(default_factory=list)  # "dense" | "moe" per layer
    dense_intermediate: int = 12288
    kda: KDAConfig = field(default_factory=KDAConfig)
    mla: MLAConfig = field(default_factory=MLAConfig)
    moe: MoEConfig = field(default_factory=MoEConfig)
    dsa: DSAConfig = field(default_factory=DSAConfig)
    gqa: GQAConfig = field(default_factory=GQAConfig)
    # per-layer n-gram embeddings (PLE) from an EXL3-coded table file: ple_heads hash heads of ple_dim
    # channels (head h hashes the last ple_orders[h] tokens into its ple_vocab rows); the rows are
    # projected to the hidden size and added to the token embedding.  ple_path "" draws a random table
    # (synthetic runs).  0 heads: none.
    ple_heads: int = 0
    ple_dim: int = 256
    ple_vocab: int = 4096
    ple_bits: int = 4
    ple_orders: list[int] = field(default_factory=list)
    ple_path: str = ""
    # Engram n-gram memory (DeepSeek-V4.1 style): at each layer of engram_layers a gated block adds the
    # projection of the token's retrieved rows to the attention output; rows come from one storage-backed
    # table of engram_heads x engram_vocab rows of engram_dim e4m3 values with E8M0 block scales, head h
    # hashing the last engram_orders[h] tokens.  engram_path "" draws a random table (synthetic runs).
    engram_layers: list[int] = field(default_factory=list)
    engram_heads: int = 4
    engram_dim: int = 256
    engram_vocab: int = 4096
    engram_orders: list[int] = field(default_factory=list)
    engram_path: str = ""
    rms_eps: float = 1e-5
    max_position: int = 1 << 20
    tie_embeddings: bool = False
    num_mtp_layers: int = 0
    dtype: str = "bfloat16"
    # manifold-constrained hyper-connections: hc_mult residual streams (0: the plain residual);
    # hc_delayed collapses each sublayer input with the previous boundary's pre (DeepSeek-V4.1 form)
    hc_mult: int = 0
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    hc_post_mult: float = 2.0
    hc_delayed: bool = False

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ["mla" if i % 4 == 3 else "kda" for i in range(self.num_layers)]
        if not self.mlp_types:
            self.mlp_types = ["moe"] * self.num_layers
        assert len(self.layer_types) == self.num_layers and len(self.mlp_types) == self.num_layers

    @property
    def num_kda_layers(self) -> int:
        return sum(t == "kda" for t in self.layer_types)

    @property
    def num_mla_layers(self) -> int:
        return sum(t == "mla" for t in self.layer_types)

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), indent=2)

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        d = dict(d)
        kda = KDAConfig(**d.pop("kda", {}))
        mla = MLAConfig(**d.pop("mla", {}))
        moe = MoEConfig(**d.pop("moe", {}))
        dsa = DSAConfig(**d.pop("dsa", {}))
        gqa = GQAConfig(**d.pop("gqa", {}))
        return ModelConfig(kda=kda, mla=mla, moe=moe, dsa=dsa, gqa=gqa, **d)


def config3() -> ModelConfig:
    """hybrid KDA/MLA MoE (EXL3 4-bit experts)."""
    return ModelConfig(
        name="hybrid-kda-mla-moe-48L-2304",
        vocab_size=163840,
        hidden_size=2304,
        num_layers=48,
        kda=KDAConfig(num_heads=32, head_dim=128),
        mla=MLAConfig(num_heads=32, q_lora_rank=768),
        moe=MoEConfig(num_experts=256, top_k=8, intermediate=1024, num_shared=1, shared_intermediate=1024,
                      router="softmax", expert_format="exl3", exl3_bits_x2=8, exl3_codebook=2),
    )


def config4() -> ModelConfig:
    """DeepSeek-style sparse-MLA MoE (Marlin int4 experts, fp8 attention)."""
    L = 43
    return ModelConfig(
        name="deepseek-sparse-mla-moe-43L-4096",
        vocab_size=129280,
        hidden_size=4096,
        num_layers=L,
        layer_types=["mla"] * L,
        mlp_types=["dense"] * 3 + ["moe"] * (L - 3),
        dense_intermediate=12288,
        mla=MLAConfig(num_heads=128, q_lora_rank=1536, attn_weight_format="fp8_block"),
        moe=MoEConfig(num_experts=256, top_k=8, intermediate=1536, num_shared=1, shared_intermediate=1536,
                      router="sigmoid", routed_scaling=2.5, expert_format="marlin"),
        num_mtp_layers=1,
    )


def config2_layer() -> ModelConfig:
    """a single sparse-MLA decode layer (128 heads)."""
    return ModelConfig(
        name="sparse-mla-decode-layer",
        vocab_size=32000,
        hidden_size=7168,
        num_layers=1,
        layer_types=["mla"],
        mlp_types=["none"],
        mla=MLAConfig(num_heads=128, q_lora_rank=1536),
    )


def tiny(layers: int = 4, experts: int = 8, hidden: int = 256, vocab: int = 512, expert_format: str = "exl3",
         layer_types: list[str] | None = None) -> ModelConfig:
    """Small model of the hybrid family for tests (CPU oracle path and GPU smoke)."""
    return ModelConfig(
        name="tiny-hybrid",
        vocab_size=vocab,
        hidden_size=hidden,
        num_layers=layers,
        layer_types=layer_types or [],
        kda=KDAConfig(num_heads=2, head_dim=128),
        mla=MLAConfig(num_heads=2, q_lora_rank=128, index_n_heads=64, index_topk=64),
        moe=MoEConfig(num_experts=experts, top_k=2, intermediate=128, num_shared=1, shared_intermediate=128,
                      expert_format=expert_format),
        max_position=4096,
    )


def tiny_deepseek(layers: int = 3, experts: int = 8, hidden: int = 256, vocab: int = 512) -> ModelConfig:
    """Small model of the DeepSeek family (all sparse-MLA, Marlin experts, fp8 attention, dense first layer)."""
    return ModelConfig(
        name="tiny-deepseek",
        vocab_size=vocab,
        hidden_size=hidden,
        num_layers=layers,
        layer_types=["mla"] * layers,
        mlp_types=["dense"] + ["moe"] * (layers - 1),
        dense_intermediate=256,
        mla=MLAConfig(num_heads=2, q_lora_rank=128, index_n_heads=64, index_topk=64, attn_weight_format="fp8_block"),
        moe=MoEConfig(num_experts=experts, top_k=2, intermediate=256, num_shared=1, shared_intermediate=128,
                      router="sigmoid", routed_scaling=2.5, expert_format="marlin"),
        max_position=4096,
        num_mtp_layers=1,
    )


def tiny_dsv4(layers: int = 3, experts: int = 8, hidden: int = 256, vocab: int = 512,
              engram: bool = False) -> ModelConfig:
    """Small DeepSeek-V4.1-style model: compressed sparse attention layers (window + ratio 1 / 2 /
    window-only), sqrt-softplus routing, EXL3 experts, delayed hyper-connections; with `engram` an
    Engram memory block at layer 1."""
    ratios = [(1, 2, 0)[i % 3] for i in range(layers)]
    return ModelConfig(
        name="tiny-dsv4",
        vocab_size=vocab,
        hidden_size=hidden,
        num_layers=layers,
        layer_types=["dsa"] * layers,
        mlp_types=["dense"] + ["moe"] * (layers - 1),
        dense_intermediate=256,
        dsa=DSAConfig(num_heads=4, q_lora_rank=128, window=16, compress_ratios=ratios, index_n_heads=4,
                      index_topk=8, index_rank_groups=2, o_groups=2, o_lora_rank=128),
        moe=MoEConfig(num_experts=experts, top_k=2, intermediate=256, num_shared=1, shared_intermediate=128,
                      router="sqrt_softplus", routed_scaling=1.5, expert_format="exl3"),
        max_position=4096,
        hc_mult=4,
        hc_delayed=True,
        engram_layers=[1] if engram and layers > 1 else [],
        engram_heads=2, engram_dim=256, engram_vocab=1024, engram_orders=[2, 3],
    )


def qwen38_flash_next() -> ModelConfig:
    """Qwen3.8-Flash-Next-style linear / full hybrid (the reference's third served family, README.md:32-37,
    vllm_sm80/models/qwen4_exp/): 48 layers at 3:1 gated-delta-net : gated full attention, hidden 2048,
    linear attention 16 query / key heads and 32 value heads of 128, full attention 16 query / 2 key-value
    heads of 256 with a 64-dim rotary part, 512 routed experts top-10 + 1 shared (intermediate 512), EXL3
    4-bit experts, a compressed n-gram PLE table, one MTP layer."""
    L = 48
    return ModelConfig(
        name="qwen-linear-full-hybrid-moe-48L-2048",
        vocab_size=151936,
        hidden_size=2048,
        num_layers=L,
        layer_types=["gqa" if i % 4 == 3 else "kda" for i in range(L)],
        kda=KDAConfig(num_heads=32, head_dim=128, mode="gdn", num_k_heads=16),
        gqa=GQAConfig(num_heads=16, num_kv_heads=2, head_dim=256, rotary_dim=64),
        moe=MoEConfig(num_experts=512, top_k=10, intermediate=512, num_shared=1, shared_intermediate=512,
                      router="softmax", expert_format="exl3", exl3_bits_x2=8, exl3_codebook=2),
        rms_eps=1e-6,
        ple_heads=4, ple_dim=256, ple_vocab=1 << 20, ple_orders=[2, 3, 2, 3],
        num_mtp_layers=1,
    )


def tiny_qwen(layers: int = 4, experts: int = 8, hidden: int = 256, vocab: int = 512, ple: bool = True) -> ModelConfig:
    """Small model of the Qwen3-Next-style family for tests."""
    return ModelConfig(
        name="tiny-qwen",
        vocab_size=vocab,
        hidden_size=hidden,
        num_layers=layers,
        layer_types=["gqa" if i % 4 == 3 else "kda" for i in range(layers)],
        kda=KDAConfig(num_heads=4, head_dim=128, mode="gdn", num_k_heads=2),
        gqa=GQAConfig(num_heads=4, num_kv_heads=2, head_dim=256, rotary_dim=64),
        moe=MoEConfig(num_experts=experts, top_k=2, intermediate=128, num_shared=1, shared_intermediate=128,
                      expert_format="exl3"),
        max_position=4096,
        ple_heads=2 if ple else 0, ple_dim=128, ple_vocab=1024, ple_orders=[2, 3],
    )


PRESETS = {"config3": config3, "config4": config4, "config2_layer": config2_layer, "tiny": tiny,
           "tiny_deepseek": tiny_deepseek, "tiny_dsv4": tiny_dsv4, "qwen38_flash_next": qwen38_flash_next,
           "tiny_qwen": tiny_qwen}


@dataclass
class ParallelConfig:
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    expert_parallel: bool = False  # experts split whole across ranks (else TP-split experts)
    fused_comm: bool = True  # product path: fused GEMM+collective kernels; False = NCCL baseline
    # with expert parallelism: steps whose tokens divide over the group keep the residual stream sharded
    # by tokens (all-gather / reduce-scatter around attention, dispatch / combine around the experts)
    sequence_parallel: bool = True

    @property
    def world_size(self) -> int:
        return self.tensor_parallel_size * self.pipeline_parallel_size


@dataclass
class SchedulerConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 8192
    # fair chunked prefill: while a running request decodes, prefill chunks of a step draw on a second
    # budget of this many tokens (0: off), split evenly between up to max_num_partial_prefills prompts
    prefill_chunk_with_decodes: int = 0
    max_num_partial_prefills: int = 1
    long_prefill_token_threshold: int = 0
    num_speculative_tokens: int = 0
    adaptive_k: str = ""  # '' off, 'by_load', 'accept' (load-adaptive draft count)
    spec_method: str = "mtp"  # drafter: 'mtp' (chained MTP head) or 'dflash' (block drafter)
    dflash_layers: int = 1  # DFlash drafter depth
    depth_policy: str = ""  # per-request verify depth policy file (dspark-depth-policy/1); "" off
    # how the policy's cut applies: "unschedule" (drafts past the depth are not verified) or "mask" (every
    # request verifies k drafts, those past its depth are masked rows: the verify step keeps one width and
    # replays its CUDA graph)
    depth_mode: str = "unschedule"
    pp_spread_decodes: bool = True  # pipeline micro-batches take equal shares of the decodes
    # asynchronous scheduling of decode steps: the next step is scheduled and launched (its input tokens
    # gathered on the device from the step in flight) before that step's tokens are read back
    async_scheduling: bool = False


@dataclass
class CacheConfig:
    block_size: int = 64
    num_blocks: int = 0  # 0: derive from memory
    gpu_memory_utilization: float = 0.90
    enable_prefix_caching: bool = False


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=config3)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    seed: int = 0
    device: str = "cuda"
    enforce_eager: bool = False
    cuda_graph_batch_sizes: list[int] = field(default_factory=lambda: [1, 2, 4, 8, 16, 32, 64, 128, 256])


def _from_hf_qwen_next(hf: dict, c: dict) -> ModelConfig:
    """Qwen3-Next-style config.json (`linear_num_key_heads`, `linear_num_value_heads`, `full_attention_interval`
    or `layer_types` of 'linear_attention' / 'full_attention', `partial_rotary_factor`, `num_experts`; the
    reference's precision switch `moe_router_dtype` and an optional PLE table)."""
    n = int(c["num_hidden_layers"])
    lt = c.get("layer_types")
    if lt:
        layer_types = ["kda" if t == "linear_attention" else "gqa" for t in lt]
    else:
        every = int(c.get("full_attention_interval", 4))
        layer_types = ["gqa" if (i + 1) % every == 0 else "kda" for i in range(n)]
    hd = int(c.get("head_dim", 256))
    kda = KDAConfig(num_heads=int(c.get("linear_num_value_heads", 32)),
                    head_dim=int(c.get("linear_value_head_dim", 128)),
                    conv_kernel=int(c.get("linear_conv_kernel_dim", 4)), mode="gdn",
                    num_k_heads=int(c.get("linear_num_key_heads", 16)))
    gqa = GQAConfig(num_heads=int(c["num_attention_heads"]), num_kv_heads=int(c.get("num_key_value_heads", 2)),
                    head_dim=hd, rotary_dim=int(hd * float(c.get("partial_rotary_factor", 0.25))),
                    rope_theta=float(c.get("rope_theta", 10000000.0)))
    moe = MoEConfig(num_experts=int(c.get("num_experts", 512)), top_k=int(c.get("num_experts_per_tok", 10)),
                    intermediate=int(c.get("moe_intermediate_size", 512)),
                    num_shared=1 if c.get("shared_expert_intermediate_size") else 0,
                    shared_intermediate=int(c.get("shared_expert_intermediate_size") or 512),
                    router="softmax", renormalize=bool(c.get("norm_topk_prob", True)),
                    router_dtype="float32" if c.get("moe_router_dtype", "float32") == "float32" else "bfloat16")
    ple = c.get("ple_config", {})
    return ModelConfig(name=str(c.get("model_type", "qwen3_next")), vocab_size=int(c["vocab_size"]),
                       hidden_size=int(c["hidden_size"]), num_layers=n, layer_types=layer_types,
                       mlp_types=["moe"] * n, kda=kda, gqa=gqa, moe=moe, rms_eps=float(c.get("rms_norm_eps", 1e-6)),
                       max_position=int(c.get("max_position_embeddings", 1 << 18)),
                       tie_embeddings=bool(hf.get("tie_word_embeddings", False)),
                       num_mtp_layers=int(c.get("num_nextn_predict_layers", c.get("mtp_num_hidden_layers", 0))),
                       ple_heads=int(ple.get("heads", 0)), ple_dim=int(ple.get("dim", 256)),
                       ple_vocab=int(ple.get("vocab", 4096)), ple_orders=list(ple.get("orders", [])),
                       ple_path=str(ple.get("path", "")))


def from_hf_config(hf: dict) -> ModelConfig:
    """ModelConfig from a Hugging Face style config.json of the supported
    families: GLM-5.x hybrid (`glm5_next[_text]`: linear_attn_config, layer_types
    'linear_attention' / 'deepseek_sparse_attention', the fixture shape of
    tests/models/fixtures/native_checkpoint_configs/glm53_flash/config.json in the
    reference) and DeepSeek-V3.x-style sparse MLA MoE (`deepseek_v3[2]`)."""
    c = hf.get("text_config", hf)
    if "linear_num_value_heads" in c or str(c.get("model_type", "")).startswith(("qwen3_next", "qwen4")):
        return _from_hf_qwen_next(hf, c)
    n = int(c["num_hidden_layers"])
    lt = c.get("layer_types")
    if lt:
        layer_types = ["kda" if t == "linear_attention" else "mla" for t in lt]
    else:
        layer_types = ["mla"] * n
    fkd = int(c.get("first_k_dense_replace", 0))
    mlp_types = c.get("mlp_layer_types")
    if mlp_types:
        mlp_types = ["moe" if t == "sparse" else "dense" for t in mlp_types]
    else:
        mlp_types = ["dense" if i < fkd else "moe" for i in range(n)]
    la = c.get("linear_attn_config", {})
    kda = KDAConfig(num_heads=int(la.get("num_heads", c.get("linear_num_heads", 32))),
                    head_dim=int(la.get("head_dim", c.get("linear_head_dim", 128))),
                    conv_kernel=int(la.get("short_conv_kernel_size", c.get("linear_conv_kernel_dim", 4))),
                    lower_bound=float(la.get("gate_lower_bound", c.get("linear_lower_bound", -5.0))))
    rope = int(c.get("qk_rope_head_dim", 64) or 64)
    mla = MLAConfig(num_heads=int(c["num_attention_heads"]), q_lora_rank=int(c.get("q_lora_rank") or 1536),
                    kv_lora_rank=int(c.get("kv_lora_rank", 512)),
                    qk_nope_head_dim=int(c.get("qk_nope_head_dim", 128)) if rope else 128,
                    qk_rope_head_dim=64, v_head_dim=min(int(c.get("v_head_dim", 128)), 512),
                    index_n_heads=int(c.get("index_n_heads", 64)), index_head_dim=int(c.get("index_head_dim", 128)),
                    index_topk=int(c.get("index_topk", 2048)), rope_theta=float(c.get("rope_theta", 10000.0)),
                    rope_interleave=bool(c.get("indexer_rope_interleave", False)))
    scoring = c.get("scoring_func", "softmax")
    moe = MoEConfig(num_experts=int(c.get("n_routed_experts", 0) or 1), top_k=int(c.get("num_experts_per_tok", 1)),
                    intermediate=int(c.get("moe_intermediate_size", c.get("intermediate_size", 1024))),
                    num_shared=int(c.get("n_shared_experts", 0) or 0),
                    shared_intermediate=int(c.get("moe_intermediate_size", 1024)),
                    router={"sigmoid": "sigmoid", "sqrtsoftplus": "sqrt_softplus"}.get(scoring, "softmax"),
                    routed_scaling=float(c.get("routed_scaling_factor", 1.0)),
                    renormalize=bool(c.get("norm_topk_prob", True)), swiglu_limit=float(c.get("swiglu_limit", 0.0)))
    return ModelConfig(name=str(c.get("model_type", "hf")), vocab_size=int(c["vocab_size"]),
                       hidden_size=int(c["hidden_size"]), num_layers=n, layer_types=layer_types, mlp_types=mlp_types,
                       dense_intermediate=int(c.get("intermediate_size", 12288)), kda=kda, mla=mla, moe=moe,
                       rms_eps=float(c.get("rms_norm_eps", 1e-5)),
                       max_position=int(c.get("max_position_embeddings", 1 << 20)),
                       tie_embeddings=bool(hf.get("tie_word_embeddings", False)),
                       num_mtp_layers=int(c.get("num_nextn_predict_layers", 0)))
