"""Failed-input isolation: a request whose step produced no valid token is finished with an error,
the rest of the batch continues.

A row whose inputs were poisoned (a NaN embedding row, the convention of
storage-backed embedding tables whose read failed after its retries) carries
NaN through every layer and the TP sums, so all of its logits are NaN; the
sampling kernels never pick a NaN (comparisons with NaN are false), leave the
row's winner at an impossible index, and the runner maps that to
``FAILED_TOKEN``.  The scheduler finishes exactly those requests with
``FINISHED_ERROR`` and frees their KV blocks and state slot, so nothing
computed from the poisoned step is reused.  No extra kernel or device
synchronisation is involved.  The reference reports failed token masks from
the worker and evicts the step's blocks
(vllm_sm80/failed_inputs.py:1-20, ``handle_failed_inputs`` :134).
"""

from __future__ import annotations

FAILED_TOKEN = -1


def sanitize(tokens: list[int], vocab_size: int) -> list[int]:
    """Map token ids outside [0, vocab_size) (no valid winner) to FAILED_TOKEN."""
    return [t if 0 <= t < vocab_size else FAILED_TOKEN for t in tokens]


def sanitize_dict(res: dict[str, list[int]], vocab_size: int) -> dict[str, list[int]]:
    return {k: sanitize(v, vocab_size) for k, v in res.items()}
