"""KDA layer core: conv + gates + gated delta rule + gated RMSNorm (one kernel on GPU)."""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import kda as _ref


def kda_forward(qkv, g_raw, beta_raw, g2, cu_seqlens, state_idx, has_init, conv_state, conv_w, conv_b, a_log, g_bias,
                lower_bound, norm_w, state, eps=1e-5, l2_eps=1e-6, out=None):
    """Varlen batch of sequences (cu_seqlens int32 [S+1]); state [slots, H, 128, 128] fp32 and
    conv_state [slots, 3*H*128, 3] bf16 are read for sequences with has_init != 0 and
    written back.  Returns [T, H*128] bf16."""
    T = qkv.shape[0]
    H = state.shape[1]
    if out is None:
        out = torch.empty(T, H * 128, dtype=torch.bfloat16, device=qkv.device)
    if not qkv.is_cuda:
        y = _ref.kda_layer(qkv, g_raw, beta_raw, g2, cu_seqlens, state, conv_state, state_idx, has_init, conv_w,
                           conv_b, a_log, g_bias, lower_bound, norm_w, eps, l2_eps)
        out.copy_(y.to(out.dtype))
        return out
    _ext.ops().kda_forward(cu_seqlens, state_idx, has_init, qkv, g_raw, beta_raw, g2, conv_state, conv_w, conv_b,
                           a_log, g_bias, lower_bound, norm_w, eps, l2_eps, 128 ** -0.5, True, state, out)
    return out
