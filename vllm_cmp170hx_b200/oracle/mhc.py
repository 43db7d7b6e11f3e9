"""fp32 oracle of manifold-constrained hyper-connections (mHC).

The residual stream is widened to `n` streams H [T, n, d].  Around every sublayer (attention, MLP):

* post (of the previous sublayer's output x): H'_k = post_k * x + sum_j comb[j, k] * H_j, rounded
  to bf16;
* coefficients of H': m = (flatten(H') @ fn^T) * rsqrt(mean(flatten(H')^2) + rms_eps) (fp32), then
  pre_k = sigmoid(s0 m_k + b_k) + eps, post_k = post_mult * sigmoid(s1 m_{n+k} + b_{n+k}),
  comb = row softmax(s2 m_{2n..} + b_{2n..}) + eps, a column normalisation, and iters - 1 more
  row/column normalisations (Sinkhorn: comb tends to a doubly stochastic matrix);
* the sublayer input: RMSNorm(bf16(sum_k mix_k H'_k)) with mix = the fresh pre ("immediate", the
  GLM-5.3 form), or the pre carried from the previous boundary (None: stream 0) -- the "delayed"
  DeepSeek-V4.1 form, which returns the fresh pre for the next boundary.

Behaviour follows the reference's formulas (vllm_sm80/models/deepseek_v41/ops/sm80_mhc.py:33-202;
GLM op contract vllm_sm80/kernels/mhc/fused_op.py:22); this is an independent implementation
used as the CPU path and as the test oracle of the fused kernel (csrc/mhc.cu).
"""

from __future__ import annotations

import torch


def coefficients(Hp: torch.Tensor, fn: torch.Tensor, scale: torch.Tensor, base: torch.Tensor, rms_eps: float,
                 eps: float, post_mult: float, iters: int):
    """Hp bf16 [T, n, d] -> pre [T, n], post [T, n], comb [T, n, n] (fp32)."""
    T, n, d = Hp.shape
    v = Hp.reshape(T, n * d).float()
    m = (v @ fn.float().t()) * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + rms_eps)
    s = scale.float()
    b = base.float()
    pre = torch.sigmoid(m[:, :n] * s[0] + b[:n]) + eps
    post = post_mult * torch.sigmoid(m[:, n:2 * n] * s[1] + b[n:2 * n])
    c = (m[:, 2 * n:] * s[2] + b[2 * n:]).view(T, n, n)
    c = torch.exp(c - c.max(dim=-1, keepdim=True).values)
    c = c / c.sum(dim=-1, keepdim=True) + eps
    c = c / (c.sum(dim=-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        c = c / (c.sum(dim=-1, keepdim=True) + eps)
        c = c / (c.sum(dim=-2, keepdim=True) + eps)
    return pre, post, c


def apply_post(x: torch.Tensor, H: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """bf16(post_k x + sum_j comb[j, k] H_j): x [T, d], H [T, n, d] -> [T, n, d]."""
    mixed = torch.einsum("tjk,tjd->tkd", comb.float(), H.float())
    return (post.float().unsqueeze(-1) * x.float().unsqueeze(1) + mixed).to(H.dtype)


def collapse_norm(Hp: torch.Tensor, mix: torch.Tensor | None, norm_w: torch.Tensor, norm_eps: float) -> torch.Tensor:
    """RMSNorm(bf16(sum_k mix_k Hp_k)); mix None selects stream 0."""
    if mix is None:
        c = Hp[:, 0]
    else:
        c = (mix.float().unsqueeze(-1) * Hp.float()).sum(1).to(Hp.dtype)
    cf = c.float()
    cf = cf * torch.rsqrt(cf.pow(2).mean(-1, keepdim=True) + norm_eps)
    return (norm_w.float() * cf).to(Hp.dtype)


def post_pre(x, H, post, comb, fn, scale, base, norm_w, *, rms_eps: float, eps: float, post_mult: float,
             iters: int, norm_eps: float, delayed: bool = False, pre_mix=None):
    """One sublayer boundary: the previous sublayer's post (skipped when x is None), the new
    coefficients, and the next sublayer's normalised input.  Returns (H', input, post, comb, pre)."""
    Hp = H if x is None else apply_post(x, H, post, comb)
    pre, post_n, comb_n = coefficients(Hp, fn, scale, base, rms_eps, eps, post_mult, iters)
    mix = pre_mix if delayed else pre
    return Hp, collapse_norm(Hp, mix, norm_w, norm_eps), post_n, comb_n, pre
