"""Host-side range checks of a step's cache and state indices (debug mode).

Before the device inputs of a step are uploaded, every slot-mapping entry,
block-table entry, recurrent-state slot and position is checked against the
sizes of the pools it indexes; a violation raises :class:`StateIndexError`
naming the request, instead of a kernel writing out of bounds.  Enabled by
``VLLM_B200_STATE_INDEX_CHECK`` (the reference's ``VLLM_STATE_INDEX_CHECK``,
vllm_sm80/worker/state_index_check.py:1-40).  It reads host arrays only, so it
costs no device synchronisation.
"""

from __future__ import annotations

import numpy as np


class StateIndexError(RuntimeError):
    pass


def check_step(h: dict, out, num_blocks: int, block_size: int, num_slots: int, max_model_len: int) -> None:
    rows = num_blocks * block_size
    slots = h["slots"]
    bad = (slots != -1) & ((slots < 0) | (slots >= rows))
    if bad.any():
        raise StateIndexError(f"slot mapping outside [0, {rows}) at tokens {np.nonzero(bad)[0][:8].tolist()}")
    bt = h["bt"]
    if ((bt < 0) | (bt >= num_blocks)).any():
        i = int(np.nonzero(((bt < 0) | (bt >= num_blocks)).any(1))[0][0])
        raise StateIndexError(f"block table row {i} ({_rid(out, i)}) outside [0, {num_blocks})")
    ks = h["kslot"]
    if num_slots and ((ks < 0) | (ks >= num_slots)).any():
        i = int(np.nonzero((ks < 0) | (ks >= num_slots))[0][0])
        raise StateIndexError(f"state slot {int(ks[i])} of {_rid(out, i)} outside [0, {num_slots})")
    pos = h["pos"]
    if (pos < 0).any() or (pos >= max_model_len).any():
        raise StateIndexError(f"positions outside [0, {max_model_len})")
    T = int(h["T"])
    if h["cu"][-1] != T or (np.diff(h["cu"]) < 0).any():
        raise StateIndexError("cu_seqlens not a non-decreasing prefix of the token count")


def _rid(out, i: int) -> str:
    try:
        return out.reqs[i].req.request_id
    except (IndexError, AttributeError):
        return f"padding row {i}"
