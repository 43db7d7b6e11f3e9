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
                lower_bound, norm_w, state, eps=1e-5, l2_eps=1e-6, out=None, verify=None, records=None, gate_mode=0):
    """Varlen batch of sequences (cu_seqlens int32 [S+1]); state [slots, H, 128, 128] fp32 and
    conv_state [slots, 3*H*128, 3] bf16 are read for sequences with has_init != 0 and
    written back -- except sequences flagged in `verify` (int32 [S]), whose state is left as it was
    and whose updates go to `records` for :func:`kda_recover`.  Returns [T, H*128] bf16.

    gate_mode 0: KDA gates (g_raw [T, H*128], per-channel decay); 1: gated delta net (g_raw [T, H],
    g_bias = dt_bias [H], one decay per head, SiLU output gate).  The chunked tensor-core prefill
    takes KDA gates only (its block-local exponents need the KDA lower bound), so gated-delta-net
    prefills run the recurrence."""
    T = qkv.shape[0]
    H = state.shape[1]
    if out is None:
        out = torch.empty(T, H * 128, dtype=torch.bfloat16, device=qkv.device)
    if not qkv.is_cuda:
        if verify is not None:
            slots = state_idx.long()
            records.snapshot = (state[slots].clone(), conv_state[slots].clone(), verify.clone())
            records.inputs = (qkv, g_raw, beta_raw, g2, cu_seqlens, state_idx, conv_w, conv_b, a_log, g_bias,
                              lower_bound, norm_w, eps, l2_eps, gate_mode)
        y = _ref.kda_layer(qkv, g_raw, beta_raw, g2, cu_seqlens, state, conv_state, state_idx, has_init, conv_w,
                           conv_b, a_log, g_bias, lower_bound, norm_w, eps, l2_eps, gate_mode=gate_mode)
        out.copy_(y.to(out.dtype))
        return out
    rec = None
    if verify is not None:
        if records.rec is None or records.rec.numel() < T * H * 3 * 128:
            records.rec = torch.empty(max(T, 1), H, 3, 128, dtype=torch.float32, device=qkv.device)
        rec = records.rec
    min_len, scratch = 0, None
    S = cu_seqlens.numel() - 1
    # a sequence can reach CHUNK_MIN_LEN tokens only if T - (S - 1) does (decode steps never launch it)
    if verify is None and not gate_mode and T - (S - 1) >= CHUNK_MIN_LEN and lower_bound >= -5.8 and _chunked_enabled():
        # sequences of at least CHUNK_MIN_LEN tokens run in chunks of 64 on the tensor cores
        min_len = CHUNK_MIN_LEN
        scratch = _chunk_scratch(T, H, qkv.device)
    _ext.ops().kda_forward(cu_seqlens, state_idx, has_init, qkv, g_raw, beta_raw, g2, conv_state, conv_w, conv_b,
                           a_log, g_bias, lower_bound, norm_w, eps, l2_eps, 128 ** -0.5, True, state, out, verify, rec,
                           min_len, scratch, _ext.status_word(qkv.device) if min_len else None, gate_mode)
    if verify is not None:
        records.inputs = (qkv, cu_seqlens, state_idx)
    return out


CHUNK_MIN_LEN = 64


def _chunked_enabled() -> bool:
    from .. import envs

    mode = envs.get("VLLM_B200_KDA_PREFILL")
    if mode not in ("chunked", "recurrent"):
        raise ValueError(f"VLLM_B200_KDA_PREFILL={mode!r}: 'chunked' or 'recurrent'")
    return mode == "chunked"


def chunk_scratch_bytes(T: int, H: int) -> int:
    """Bytes of the chunked prefill's per-token inputs (q, k, v bf16 and the log2 decay fp32 per
    channel, beta per head), as the kernel lays them out."""
    n = T * H * 128
    return n * 10 + T * H * 4 + 1280


def _chunk_scratch(T: int, H: int, dev) -> torch.Tensor:
    return torch.empty(chunk_scratch_bytes(T, H), dtype=torch.uint8, device=dev)


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
    (qkv, g_raw, beta_raw, g2, cu, sidx, conv_w, conv_b, a_log, g_bias, lb, norm_w, eps, l2_eps, gm) = records.inputs
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
                       eps, l2_eps, gate_mode=gm)
