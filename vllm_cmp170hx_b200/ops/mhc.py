"""Manifold-constrained hyper-connections (mHC): one fused op per sublayer boundary.

`post_pre` applies the previous sublayer's post to the residual streams, computes the streams'
new coefficients (pre / post / Sinkhorn-normalised comb) and produces the next sublayer's
normalised input -- on the GPU in one kernel (csrc/mhc.cu, one CTA per token), on CPU tensors
with the fp32 oracle (oracle/mhc.py).  The reference runs the same contract as its fused decode
kernel (vllm_sm80/kernels/mhc/decode.py:865) and, for DeepSeek-V4.1, as the delayed variant
(vllm_sm80/models/deepseek_v41/ops/sm80_mhc.py:158).
"""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import mhc as _ref


def post_pre(x: torch.Tensor | None, H: torch.Tensor, post: torch.Tensor | None, comb: torch.Tensor | None,
             fn: torch.Tensor, scale: torch.Tensor, base: torch.Tensor, norm_w: torch.Tensor, *, rms_eps: float,
             eps: float, post_mult: float, iters: int, norm_eps: float, delayed: bool = False,
             pre_mix: torch.Tensor | None = None):
    """x [T, d] bf16 (the previous sublayer's output; None: no post), H [T, n, d] bf16 streams,
    post [T, n] / comb [T, n, n] fp32 (the previous boundary's), fn [2n + n^2, n d] fp32,
    scale [3], base [2n + n^2] fp32, norm_w [d] bf16.  Returns (H', input [T, d] bf16, post, comb,
    pre) with H' written over H on the GPU (in place)."""
    if not H.is_cuda:
        return _ref.post_pre(x, H, post, comb, fn, scale, base, norm_w, rms_eps=rms_eps, eps=eps,
                             post_mult=post_mult, iters=iters, norm_eps=norm_eps, delayed=delayed, pre_mix=pre_mix)
    T, n, d = H.shape
    dev = H.device
    y = torch.empty(T, d, dtype=H.dtype, device=dev)
    post_o = torch.empty(T, n, dtype=torch.float32, device=dev)
    comb_o = torch.empty(T, n, n, dtype=torch.float32, device=dev)
    pre_o = torch.empty(T, n, dtype=torch.float32, device=dev)
    mode = 0 if not delayed else (1 if pre_mix is not None else 2)
    _ext.ops().mhc_post_pre(x, H, post, comb, fn, scale, base, norm_w, pre_mix, float(rms_eps), float(eps),
                            float(post_mult), int(iters), float(norm_eps), mode, H, y, post_o, comb_o, pre_o)
    return H, y, post_o, comb_o, pre_o
