"""KDA layer core: conv + gates + gated delta rule + gated RMSNorm (one kernel on GPU)."""

from __future__ import annotations

import torch

from .. import _ext
from ..oracle import kda as _ref


class KdaRecords:
    """What a speculative verify step leaves for :func:`kda_recover` of one KDA layer.  GPU: the
    per-token (u, k, decay) records [T, H, 3, 128] written by the kernel (the reference's RecoverSSM
    records, vllm_sm80/kernels/kda/recover.py:1-40).  CPU oracle: the verified sequences' states and
    conv windows from before the step, and the step's inputs, to re-run the kept prefix."""

    def __init__(self):
        self.rec = None
        self.snapshot = None
        self.inputs = None


def kda_forward(qkv, g_raw, beta_raw, g2, cu_seqlens, state_idx, has_init, conv_state, conv_w, conv_b, a_log, g_bias,
                lower_bound, norm_w, state, eps=1e-5, l2_eps=1e-6, out=None, verify=None, records=None):
    """Varlen batch of sequences (cu_seqlens int32 [S+1]); state [slots, H, 128, 128] fp32 and
    conv_state [slots, 3*H*128, 3] bf16 are read for sequences with has_init != 0 and
    written back -- except sequences flagged in `verify` (int32 [S]), whose state is left as it was
    and whose updates go to `records` for :func:`kda_recover`.  Returns [T, H*128] bf16."""
    T = qkv.shape[0]
    H = state.shape[1]
    if out is None:
        out = torch.empty(T, H * 128, dtype=torch.bfloat16, device=qkv.device)
    if not qkv.is_cuda:
        if verify is not None:
            slots = state_idx.long()
            records.snapshot = (state[slots].clone(), conv_state[slots].clone(), verify.clone())
            records.inputs = (qkv, g_raw, beta_raw, g2, cu_seqlens, state_idx, conv_w, conv_b, a_log, g_bias,
                              lower_bound, norm_w, eps, l2_eps)
        y = _ref.kda_layer(qkv, g_raw, beta_raw, g2, cu_seqlens, state, conv_state, state_idx, has_init, conv_w,
                           conv_b, a_log, g_bias, lower_bound, norm_w, eps, l2_eps)
        out.copy_(y.to(out.dtype))
        return out
    rec = None
    if verify is not None:
        if records.rec is None or records.rec.numel() < T * H * 3 * 128:
            records.rec = torch.empty(max(T, 1), H, 3, 128, dtype=torch.float32, device=qkv.device)
        rec = records.rec
    _ext.ops().kda_forward(cu_seqlens, state_idx, has_init, qkv, g_raw, beta_raw, g2, conv_state, conv_w, conv_b,
                           a_log, g_bias, lower_bound, norm_w, eps, l2_eps, 128 ** -0.5, True, state, out, verify, rec)
    if verify is not None:
        records.inputs = (qkv, cu_seqlens, state_idx)
    return out


def kda_recover(records: KdaRecords, keep: torch.Tensor, state: torch.Tensor, conv_state: torch.Tensor) -> None:
    """Bring every verified sequence's state and conv window to the end of its first keep[s] tokens
    (keep: int32 [S]; 0 leaves a sequence as it is)."""
    if records.rec is not None:
        qkv, cu, sidx = records.inputs
        _ext.ops().kda_recover(cu, sidx, keep.to(device=qkv.device, dtype=torch.int32), records.rec, state, qkv,
                               conv_state)
        return
    if records.snapshot is None:
        return
    (qkv, g_raw, beta_raw, g2, cu, sidx, conv_w, conv_b, a_log, g_bias, lb, norm_w, eps, l2_eps) = records.inputs
    st0, cv0, verify = records.snapshot
    cu_l = cu.tolist()
    for s in range(len(cu_l) - 1):
        n = int(keep[s])
        if not int(verify[s]) or n <= 0:
            continue
        slot = int(sidx[s])
        state[slot] = st0[s]
        conv_state[slot] = cv0[s]
        a, b = cu_l[s], cu_l[s] + n
        one = torch.tensor([0, n], dtype=torch.int32)
        _ref.kda_layer(qkv[a:b], g_raw[a:b], beta_raw[a:b], None if g2 is None else g2[a:b], one, state, conv_state,
                       sidx[s:s + 1], torch.ones(1, dtype=torch.int32), conv_w, conv_b, a_log, g_bias, lb, norm_w,
                       eps, l2_eps)
