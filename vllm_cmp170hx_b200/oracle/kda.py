"""KDA (gated delta rule with per-channel decay) references.

* :func:`naive_recurrence` -- token-sequential recurrence, the definition
  (tests/kernels/test_ampere_pp_kda_prefill.py:228-248 of the reference):
  ``S <- S * e_t; u = (v_t - S k_t) * beta_t; S <- S + u k_t^T; o_t = S q_t``
  with S in R^{V x K} and e_t = exp(g_t) broadcast over rows.
* :func:`chunked` -- the same result computed chunk-parallel (UT form): per
  chunk of C tokens, with cumulative log-decay G_t,
  ``U = (I + diag(beta) L)^{-1} diag(beta) (V - S0 (K*exp(G))^T)``,
  ``L[s, r] = sum_k k_s k_r exp(G_s - G_r)`` (r < s),
  ``o_t = S0 (q_t*exp(G_t)) + sum_{s<=t} u_s (sum_k k_s q_t exp(G_t - G_s))``,
  ``S_C = S0 diag(exp(G_C)) + sum_s u_s (k_s*exp(G_C - G_s))^T``.
  Every exponent is of a non-positive number, so the form is stable without
  a lower bound on the decay.
* :func:`kda_layer` -- the GLM KDA layer core for a varlen batch: causal
  conv1d (kernel 4) + SiLU on q/k/v, L2 norm, decay gate
  ``exp(lb * sigmoid(exp(A_log) * (g + bias)))``, recurrence, gated RMSNorm
  with ``sigmoid(g2)`` (vllm_sm80/models/glm5next/ops/kda_decode.py:1-60).
"""

from __future__ import annotations

import torch


def naive_recurrence(q, k, v, g, beta, S0=None):
    """q, k, v, g: [B, T, H, D]; beta: [B, T, H]; S0: [B, H, D, D] or None.
    Returns (o [B, T, H, D], S [B, H, D, D]) in the inputs' dtype."""
    B, T, H, D = q.shape
    S = torch.zeros(B, H, D, D, dtype=q.dtype) if S0 is None else S0.clone()
    o = torch.empty_like(v)
    for t in range(T):
        S = S * torch.exp(g[:, t])[:, :, None, :]
        kv = torch.einsum("bhvk,bhk->bhv", S, k[:, t])
        u = (v[:, t] - kv) * beta[:, t, :, None]
        S = S + u[..., :, None] * k[:, t][..., None, :]
        o[:, t] = torch.einsum("bhvk,bhk->bhv", S, q[:, t])
    return o, S


def chunked(q, k, v, g, beta, S0=None, chunk: int = 64):
    """Chunk-parallel evaluation of the same recurrence (see module doc)."""
    B, T, H, D = q.shape
    dt = q.dtype
    S = torch.zeros(B, H, D, D, dtype=dt) if S0 is None else S0.clone()
    o = torch.empty_like(v)
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        C = c1 - c0
        qc, kc, vc = (x[:, c0:c1].permute(0, 2, 1, 3) for x in (q, k, v))  # [B, H, C, D]
        bc = beta[:, c0:c1].permute(0, 2, 1)  # [B, H, C]
        G = torch.cumsum(g[:, c0:c1].permute(0, 2, 1, 3), dim=2)  # [B, H, C, D]
        # pairwise decays exp(G_s - G_r) for r <= s (masked elsewhere)
        diff = G[:, :, :, None, :] - G[:, :, None, :, :]  # [B, H, s, r, D]
        tri = torch.tril(torch.ones(C, C, dtype=torch.bool))
        dec = torch.where(tri[None, None, :, :, None], torch.exp(diff.clamp(max=0)), torch.zeros((), dtype=dt))
        L = torch.einsum("bhsd,bhrd,bhsrd->bhsr", kc, kc, dec)
        L = L * torch.tril(torch.ones(C, C, dtype=dt), -1)
        A = kc * torch.exp(G)  # a_s = k_s * exp(G_s)
        rhs = bc[..., None] * (vc - torch.einsum("bhvk,bhsk->bhsv", S, A))
        Tm = torch.eye(C, dtype=dt) + bc[..., None] * L
        U = torch.linalg.solve_triangular(Tm, rhs, upper=False, unitriangular=False)
        cq = qc * torch.exp(G)
        inner = torch.einsum("bhsd,bhtd,bhtsd->bhts", kc, qc, dec)  # s <= t
        oc = torch.einsum("bhvk,bhtk->bhtv", S, cq) + torch.einsum("bhts,bhsv->bhtv", inner, U)
        o[:, c0:c1] = oc.permute(0, 2, 1, 3)
        GC = G[:, :, -1:, :]  # [B, H, 1, D]
        kend = kc * torch.exp(GC - G)
        S = S * torch.exp(GC)[:, :, 0, None, :] + torch.einsum("bhsv,bhsk->bhvk", U, kend)
    return o, S


def conv_silu(x, w, b, state):
    """Causal depthwise conv (kernel 4) + SiLU of one sequence.  x: [T, C];
    w: [C, 4]; state: [C, 3] previous inputs (oldest first).  Returns (y, new_state)."""
    full = torch.cat([state.t().float(), x.float()], dim=0)  # [T+3, C]
    T = x.shape[0]
    y = torch.zeros(T, x.shape[1], dtype=torch.float32)
    for i in range(4):
        y += full[i:i + T] * w[:, i].float()
    if b is not None:
        y += b.float()
    y = torch.nn.functional.silu(y)
    return y, full[-3:].t().contiguous()


def kda_layer(qkv, g_raw, beta_raw, g2, cu_seqlens, state, conv_state, state_idx, has_init, conv_w, conv_b, a_log,
              g_bias, lower_bound, norm_w, eps=1e-5, l2_eps=1e-6, round_conv=True, gate_mode=0):
    """Varlen GLM KDA layer core (fp32 math).  Shapes as the CUDA op
    `kda_forward`.  Updates state / conv_state in place; returns out [T, H*D] fp32.

    gate_mode 1 is the gated delta net of Qwen3-Next-style linear attention: g_raw [T, H] and g_bias
    [H] (dt_bias) give one log decay per head, -exp(A_log) * softplus(g + dt_bias), broadcast over the
    key channels, and the output gate is silu(g2) instead of sigmoid(g2)."""
    H = state.shape[1]
    D = 128
    HD = H * D
    T = qkv.shape[0]
    out = torch.zeros(T, HD, dtype=torch.float32)
    for s in range(len(cu_seqlens) - 1):
        t0, t1 = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        slot = int(state_idx[s]) if state_idx is not None else s
        init = bool(has_init[s]) if has_init is not None else True
        if t1 == t0:
            continue
        cs = conv_state[slot] if init else torch.zeros_like(conv_state[slot])
        y, new_cs = conv_silu(qkv[t0:t1, : 3 * HD], conv_w, conv_b, cs)
        if round_conv:
            y = y.to(torch.bfloat16).float()
        conv_state[slot] = new_cs.to(conv_state.dtype)
        q = y[:, :HD].view(-1, H, D)
        k = y[:, HD:2 * HD].view(-1, H, D)
        v = y[:, 2 * HD:].view(-1, H, D)
        q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + l2_eps) * D ** -0.5
        k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + l2_eps)
        a = torch.exp(a_log.float())[:, None]
        if gate_mode:
            x = g_raw[t0:t1, :H].float() + (g_bias.float().view(H) if g_bias is not None else 0)
            g = (-a[:, 0] * torch.nn.functional.softplus(x))[..., None].expand(-1, H, D)  # log decay per head
        else:
            x = g_raw[t0:t1].float().view(-1, H, D) + (g_bias.float().view(H, D) if g_bias is not None else 0)
            g = lower_bound * torch.sigmoid(a * x)  # log decay
        beta = torch.sigmoid(beta_raw[t0:t1].float().view(-1, H))
        S0 = state[slot].float()[None] if init else None
        o, S = naive_recurrence(q[None], k[None], v[None], g[None], beta[None], S0)
        state[slot] = S[0].to(state.dtype)
        o = o[0]
        if norm_w is not None:
            o = o * torch.rsqrt((o * o).mean(-1, keepdim=True) + eps) * norm_w.float()
            if g2 is not None:
                z = g2[t0:t1].float().view(-1, H, D)
                o = o * (torch.nn.functional.silu(z) if gate_mode else torch.sigmoid(z))
        out[t0:t1] = o.reshape(-1, HD)
    return out
