"""Per-request verification depth: how many of a request's drafts are worth verifying.

A policy file (schema ``dspark-depth-policy/1``, the reference's format, kept alike so existing
policy files load: vllm_sm80/spec_decode/dspark_row_mask.py:18-64, decision rule
dspark_row_mask_kernel.py:6-33)::

    {"schema": "dspark-depth-policy/1", "max_depth": 7,
     "features": ["bias", "logit_conf", "logit_top1", "ent"],
     "weights": [[w per feature] for draft positions 1 .. max_depth],
     "costs": {"<batch>": {"<k>": ms, ...}, ...},
     "tau": {"<batch>": threshold, ...}}          (optional)

Draft position i (1-based) gets the acceptance estimate p_i = sigmoid(sum_f w[i-1][f] x_f) over
the listed features: bias (1), logit_conf (log-odds of a confidence head's output), logit_top1
(log-odds of the draft distribution's top-1 probability) and ent (its entropy in nats), with
probabilities clamped to [1e-6, 1 - 1e-6] before the log-odds.  For a step of b requests each
verifying up to K drafts:

    E(k)     = 1 + sum_{i <= k} prod_{j <= i} p_j                 (expected tokens emitted)
    cost(k)  = T_b(K) - (T_b(K) - T_b(k)) / b                     (this request's share)
    live     = argmax_{k = 0..K} E(k) / cost(k)   (ties: the larger k)
    or, with a tau for b >= 2: the largest k with prod_{j <= k} p_j >= tau_b (0 if none).

T_b(k) is the measured step time of b requests verifying k drafts each; batch sizes the file does
not list are interpolated linearly between the nearest listed ones (the nearest one outside them),
tau likewise.  The reference keeps every request's K + 1 verify rows (uniform CUDA-graph shapes)
and makes the rows past `live` skip the routed experts; the speculative path here is eager, so
the drafts past `live` are simply not scheduled -- their rows are never computed, and greedy
output equals the unmasked output truncated at `live`.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass

import torch

SCHEMA = "dspark-depth-policy/1"
FEATURES = ("bias", "logit_conf", "logit_top1", "ent")
PROB_EPS = 1e-6


def _interp(table: dict[int, float], b: int) -> float:
    keys = sorted(table)
    if b <= keys[0]:
        return table[keys[0]]
    if b >= keys[-1]:
        return table[keys[-1]]
    for lo, hi in zip(keys, keys[1:]):
        if lo <= b <= hi:
            f = (b - lo) / (hi - lo)
            return table[lo] * (1 - f) + table[hi] * f
    raise AssertionError


@dataclass(frozen=True)
class HostWidth:
    """The policy's optional ``host_width`` block: the verify width K of a decode step of b requests
    (b in ``batch_sizes``), chosen on the host from each request's p_i of its verify round
    ``lag_rounds`` back (the reference's DSpark host width, vllm_sm80/spec_decode/dspark_host_width.py:
    1-31; same block format so policy files load unchanged).  K in ``k_choices`` maximises

        sum_r E(q_r, d_r(K)) / T(b, K | d)
        d_r(K)      = the largest k <= K with prod_{j <= k} q_rj >= tau[b]   (0 if none)
        E(q, d)     = 1 + sum_{i <= d} prod_{j <= i} q_j
        T(b, K | d) = t0_ms[b] + b cum_ms[b][K] - (1 - s[b][K]) sum_r (cum_ms[b][K] - cum_ms[b][d_r])

    ties to the smaller K; ``fallback_k`` when a request has no such round."""

    batch_sizes: frozenset
    lag: int
    fallback_k: int
    k_choices: tuple  # ascending
    t0: dict
    cum: dict  # b -> (cum_ms at k = 0 .. max K)
    share: dict  # b -> {K: s}
    tau: dict

    @staticmethod
    def parse(raw: dict, where: str = "policy") -> "HostWidth":
        block = raw.get("host_width")
        if not isinstance(block, dict):
            raise ValueError(f"{where}: host_width must be an object")
        if block.get("estimate") != "stale":
            raise ValueError(f"{where}: host_width estimate must be 'stale' (p_i of an earlier round)")

        def ints(name):
            v = block.get(name)
            if (not isinstance(v, list) or not v or len(set(v)) != len(v)
                    or any(not isinstance(x, int) or isinstance(x, bool) or x < 1 for x in v)):
                raise ValueError(f"{where}: host_width {name} must be distinct positive integers: {v!r}")
            return tuple(sorted(v))

        def num(name, v):
            try:
                f = float(v)
            except (TypeError, ValueError):
                raise ValueError(f"{where}: host_width {name} is not a number: {v!r}") from None
            if not math.isfinite(f):
                raise ValueError(f"{where}: host_width {name} is not finite: {v!r}")
            return f

        lag = block.get("lag_rounds")
        if not isinstance(lag, int) or isinstance(lag, bool) or lag < 1:
            raise ValueError(f"{where}: host_width lag_rounds must be a positive integer: {lag!r}")
        ks = ints("k_choices")
        if block.get("fallback_k") not in ks:
            raise ValueError(f"{where}: host_width fallback_k must be one of k_choices {list(ks)}")
        sizes = ints("batch_sizes")
        if sizes[0] < 2:
            raise ValueError(f"{where}: host_width batch_sizes start at 2")
        raw_tau = raw.get("tau")
        if not isinstance(raw_tau, dict):
            raise ValueError(f"{where}: host_width needs the policy's tau")
        t0, cum, share, tau = {}, {}, {}, {}
        for b in sizes:
            key = str(b)
            try:
                t0_b, cum_b, s_b, tau_b = block["t0_ms"][key], block["cum_ms"][key], block["s"][key], raw_tau[key]
            except (KeyError, TypeError):
                raise ValueError(f"{where}: host_width needs t0_ms, cum_ms, s and tau at batch size {b}") from None
            tau[b] = num(f"tau[{b}]", tau_b)
            t0[b] = num(f"t0_ms[{b}]", t0_b)
            if not 0.0 < tau[b] <= 1.0 or t0[b] <= 0.0:
                raise ValueError(f"{where}: host_width tau[{b}] must be in (0, 1] and t0_ms[{b}] positive")
            if not isinstance(cum_b, list) or len(cum_b) <= ks[-1]:
                raise ValueError(f"{where}: host_width cum_ms[{b}] needs k = 0 .. {ks[-1]}")
            row = tuple(num(f"cum_ms[{b}]", v) for v in cum_b)
            if row[0] != 0.0 or any(x > y for x, y in zip(row, row[1:])):
                raise ValueError(f"{where}: host_width cum_ms[{b}] must start at 0 and not decrease")
            cum[b] = row
            if not isinstance(s_b, dict) or any(str(k) not in s_b for k in ks):
                raise ValueError(f"{where}: host_width s[{b}] needs a share for every K of k_choices")
            share[b] = {k: num(f"s[{b}][{k}]", s_b[str(k)]) for k in ks}
            if any(not 0.0 <= v <= 1.0 for v in share[b].values()):
                raise ValueError(f"{where}: host_width s[{b}] shares must be in [0, 1]")
        return HostWidth(frozenset(sizes), lag, block["fallback_k"], ks, t0, cum, share, tau)

    def choose(self, q_rows: list, b: int, cap: int) -> int | None:
        """The step's K (at most ``cap``) from each request's p_i row, ``fallback_k`` when a row is
        missing; None when b is not a batch size of the block (the width stays as it is)."""
        if b not in self.batch_sizes:
            return None
        ks = [k for k in self.k_choices if k <= cap] or [self.k_choices[0]]
        if any(q is None or len(q) < ks[-1] for q in q_rows):
            return min(self.fallback_k, cap)
        tau, cum = self.tau[b], self.cum[b]
        best, best_k = -1.0, ks[0]
        for K in ks:
            e_sum, gap = 0.0, 0.0
            for q in q_rows:
                prod, d, e = 1.0, 0, 1.0
                for j in range(K):
                    prod *= q[j]
                    if prod >= tau:
                        d = j + 1
                pp = 1.0
                for j in range(d):
                    pp *= q[j]
                    e += pp
                e_sum += e
                gap += cum[K] - cum[d]
            t = self.t0[b] + b * cum[K] - (1.0 - self.share[b][K]) * gap
            score = e_sum / t
            if score > best + 1e-12:  # ties keep the smaller K
                best, best_k = score, K
        return best_k


@dataclass
class DepthPolicy:
    weights: torch.Tensor  # [max_depth, len(FEATURES)] fp32, unlisted features 0
    costs: dict[int, list[float]]  # batch -> T_b(0..m) ms
    tau: dict[int, float]
    uses_conf: bool
    uses_stats: bool
    host_width: HostWidth | None = None

    @property
    def max_depth(self) -> int:
        return self.weights.shape[0]

    @staticmethod
    def load(path: str) -> "DepthPolicy":
        with open(path) as f:
            raw = json.load(f)
        return DepthPolicy.from_dict(raw, path)

    @staticmethod
    def from_dict(raw: dict, where: str = "policy") -> "DepthPolicy":
        if raw.get("schema") != SCHEMA:
            raise ValueError(f"{where}: schema must be {SCHEMA!r}")
        feats = raw.get("features")
        if not feats or any(f not in FEATURES for f in feats) or len(set(feats)) != len(feats):
            raise ValueError(f"{where}: features must be distinct names from {FEATURES}")
        depth = int(raw.get("max_depth", 0))
        w = raw.get("weights")
        if depth < 1 or not isinstance(w, list) or len(w) != depth or any(len(r) != len(feats) for r in w):
            raise ValueError(f"{where}: weights must be max_depth rows of one weight per feature")
        W = torch.zeros(depth, len(FEATURES), dtype=torch.float32)
        for i, row in enumerate(w):
            for f, v in zip(feats, row):
                W[i, FEATURES.index(f)] = float(v)
        costs: dict[int, list[float]] = {}
        for key, by_k in (raw.get("costs") or {}).items():
            b = int(key)
            ks = sorted(int(k) for k in by_k)
            if b < 1 or ks != list(range(len(ks))):
                raise ValueError(f"{where}: costs of batch {key} must list k = 0 .. m")
            row = [float(by_k[str(k)] if str(k) in by_k else by_k[k]) for k in ks]
            if any(v <= 0 for v in row) or any(b2 < a2 for a2, b2 in zip(row, row[1:])):
                raise ValueError(f"{where}: costs of batch {b} must be positive and nondecreasing in k")
            costs[b] = row
        if not costs:
            raise ValueError(f"{where}: costs must not be empty")
        tau = {int(k): float(v) for k, v in (raw.get("tau") or {}).items()}
        hw = HostWidth.parse(raw, where) if "host_width" in raw else None
        return DepthPolicy(W, costs, tau, "logit_conf" in feats, bool({"logit_top1", "ent"} & set(feats)), hw)

    def cost_row(self, b: int, K: int) -> list[float]:
        """T_b(0..K), interpolated over batch sizes on the k every neighbour lists."""
        keys = sorted(self.costs)
        lo = max([k for k in keys if k <= b], default=keys[0])
        hi = min([k for k in keys if k >= b], default=keys[-1])
        rows = {lo: self.costs[lo], hi: self.costs[hi]}
        m = min(len(r) for r in rows.values())
        if K >= m:
            raise ValueError(f"the policy prices at most {m - 1} drafts at batch {b}, asked {K}")
        return [_interp({k: r[i] for k, r in rows.items()}, b) for i in range(K + 1)]

    def tau_at(self, b: int) -> float:
        if b < 2 or not self.tau:
            return 0.0
        return _interp(self.tau, b)

    def accept_probs(self, feats: torch.Tensor) -> torch.Tensor:
        """feats [A, K, len(FEATURES)] -> p [A, K]."""
        K = feats.shape[1]
        w = self.weights[:K].to(feats.device)
        return torch.sigmoid((feats.float() * w[None]).sum(-1))

    def live(self, p: torch.Tensor, b: int) -> list[int]:
        """Verified depth per request from p [A, K]."""
        A, K = p.shape
        if K == 0:
            return [0] * A
        cp = torch.cumprod(p.double().cpu(), dim=1)
        tau = self.tau_at(b)
        if tau > 0:
            ok = cp >= tau
            return [int(ok[a].nonzero().max()) + 1 if ok[a].any() else 0 for a in range(A)]
        T = self.cost_row(b, K)
        cost = torch.tensor([T[K] - (T[K] - T[k]) / b for k in range(K + 1)], dtype=torch.float64)
        E = torch.cat([torch.ones(A, 1, dtype=torch.float64), 1 + cp.cumsum(1)], 1)
        ratio = E / cost[None]
        # ties go to the larger k: the last maximum
        return [K - int(torch.argmax(ratio[a].flip(0))) for a in range(A)]


def _logit(q: torch.Tensor) -> torch.Tensor:
    q = q.clamp(PROB_EPS, 1 - PROB_EPS)
    return torch.log(q) - torch.log1p(-q)


def draft_features(A: int, K: int, stats: torch.Tensor | None = None, conf: torch.Tensor | None = None,
                   device=None) -> torch.Tensor:
    """stats [A, K, 2] (top-1 probability, entropy) and conf [A, K] -> features [A, K, 4]."""
    f = torch.zeros(A, K, len(FEATURES), dtype=torch.float32, device=device)
    f[..., 0] = 1.0
    if conf is not None:
        f[..., 1] = _logit(conf.float())
    if stats is not None:
        f[..., 2] = _logit(stats[..., 0].float())
        f[..., 3] = stats[..., 1].float()
    return f


def logit_stats(logits: torch.Tensor, all_reduce=None) -> torch.Tensor:
    """Top-1 probability and entropy (nats) of softmax(logits) over the full vocabulary from this
    rank's shard [A, V_local]: the shard maxima, normalisers and sum p * logit are combined by
    `all_reduce(x, op)` (None: one shard).  Returns [A, 2] fp32."""
    import torch.distributed as dist

    x = logits.float()
    m = x.max(-1).values
    if all_reduce is not None:
        m = all_reduce(m.contiguous(), dist.ReduceOp.MAX)
    e = torch.exp(x - m[:, None])
    zs = torch.stack([e.sum(-1), (e * (x - m[:, None])).sum(-1)], 1)
    if all_reduce is not None:
        zs = all_reduce(zs.contiguous(), dist.ReduceOp.SUM)
    Z, S = zs[:, 0], zs[:, 1]
    return torch.stack([1.0 / Z, torch.log(Z) - S / Z], 1)


def describe(pol: DepthPolicy) -> str:
    return (f"depth policy: max_depth {pol.max_depth}, costs for batches {sorted(pol.costs)}, "
            f"tau {'on' if pol.tau else 'off'}, features {'conf ' if pol.uses_conf else ''}"
            f"{'stats' if pol.uses_stats else ''}".rstrip())

