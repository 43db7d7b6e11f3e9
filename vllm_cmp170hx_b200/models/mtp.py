"""Multi-token-prediction (MTP) draft head of the DeepSeek family.

One extra decoder layer predicts the token after next from
``eh_proj([RMSNorm(embed(token_{i+1})) | RMSNorm(h_i)])`` where h_i is the
target model's final hidden state at position i; the head shares the target's
embedding and (vocab-parallel) LM head.  Chained k times it proposes k draft
tokens (the upstream `num_nextn_predict_layers` drafter the reference's
config 5 uses).  Its attention layer keeps its own paged latent cache, laid
out on the same blocks as the target's (same slot mapping).
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import ModelConfig
from ..parallel import state as pstate
from .hybrid import DecoderLayer, HybridForCausalLM, StepContext
from .layers import Linear, RMSNorm, WeightInit, default_std


class MTPHead(nn.Module):
    def __init__(self, cfg: ModelConfig, target: HybridForCausalLM, device, seed: int = 0, init_mode: str = "local"):
        super().__init__()
        st = pstate.get()
        wi = WeightInit(seed + 7777, device, init_mode)
        H = cfg.hidden_size
        self.layer_id = cfg.num_layers  # cache key of the MTP layer
        # the MTP layer is an MLA layer with the model's MLP type of the last layer
        # (a plain residual inside the MTP layer even when the target widens its residual into
        # hyper-connection streams: the head consumes the target's final, collapsed hidden state)
        # (models whose full attention is gated grouped-query attention -- the Qwen3-Next-style family --
        # get an MTP layer of that kind instead, with its own paged [k | v] cache)
        self.kind = "gqa" if ("gqa" in cfg.layer_types and "mla" not in cfg.layer_types) else "mla"
        mcfg = ModelConfig.from_dict({**_cfg_dict(cfg), "num_layers": cfg.num_layers + 1, "hc_mult": 0,
                                      "layer_types": cfg.layer_types + [self.kind], "ple_heads": 0,
                                      "mlp_types": cfg.mlp_types + [cfg.mlp_types[-1]]})
        self.enorm = RMSNorm(wi.ones_plus(H, 0.05), cfg.rms_eps)
        self.hnorm = RMSNorm(wi.ones_plus(H, 0.05), cfg.rms_eps)
        self.eh_proj = Linear(wi.normal((H, 2 * H), default_std(2 * H)))
        self.layer = DecoderLayer(mcfg, self.layer_id, wi, st.tp_size, st.tp_rank)
        self.norm = RMSNorm(wi.ones_plus(H, 0.05), cfg.rms_eps)
        self.target = [target]  # not a submodule: weights are shared

    def forward(self, input_ids: torch.Tensor, prev_hidden: torch.Tensor, ctx: StepContext) -> torch.Tensor:
        t = self.target[0]
        e = self.enorm(t.embed[input_ids])
        h = self.hnorm(prev_hidden)
        x = self.eh_proj(torch.cat([e, h], dim=-1))
        x, residual = self.layer(x, None, ctx)
        return self.norm(x, residual)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.target[0].compute_logits(hidden)


def _cfg_dict(cfg: ModelConfig) -> dict:
    import dataclasses

    return dataclasses.asdict(cfg)
