"""Agreement of the per-step logits of two runs of the same requests (a parallel layout against one
device), robust to the routing near-ties of mixture-of-experts models.

A different rounding of a partial sum (another reduction order over the ranks) can move a router
logit across a near-tie and pick another expert for a token; that token's hidden state, the later
tokens of its sequence and, once a different token is sampled, the rest of that sequence then differ
by far more than the rounding.  So the check is per row (row i of every step being request i), with
the sequences that already sampled a different token left out of the later steps, and a quarter of
the remaining rows allowed to differ."""

from __future__ import annotations

import numpy as np


def step_logits_agree(got: list, ref: list, row_tol: float = 5e-2, median_tol: float = 2e-2,
                      min_frac: float = 0.75) -> tuple[bool, list]:
    """got / ref: per step, logits [rows, vocab] (numpy or torch).  Returns (ok, per-step report of
    (kept rows, row errors, rows whose greedy token differs))."""
    diverged: set[int] = set()
    report = []
    ok = len(got) == len(ref)
    for a, b in zip(got, ref):
        a = np.asarray(a, dtype=np.float64)
        b = np.asarray(b, dtype=np.float64)
        if a.shape != b.shape:
            return False, report + [("shape", a.shape, b.shape)]
        rows = [i for i in range(a.shape[0]) if i not in diverged]
        err = [float(np.linalg.norm(a[i] - b[i]) / max(np.linalg.norm(b[i]), 1e-12)) for i in rows]
        flips = [i for i in range(a.shape[0]) if int(a[i].argmax()) != int(b[i].argmax())]
        if rows:
            good = sum(e < row_tol for e in err)
            ok = ok and good >= min_frac * len(rows) and float(np.median(err)) < median_tol
        report.append((rows, [round(e, 4) for e in err], flips))
        diverged.update(flips)
    return ok, report
