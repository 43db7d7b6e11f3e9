"""Load-adaptive draft count for speculative decoding.

Policies (``SchedulerConfig.adaptive_k`` / ``VLLM_B200_ADAPTIVE_K``):

* ``by_load``: the draft count falls as the batch grows -- drafts are nearly
  free while a decode step is bound by weight streaming and cost a full token
  each once the step is compute-bound.  A table of (max running requests, k)
  rows, the first row whose bound holds wins.
* ``accept``: pick k maximising expected tokens per unit step cost,
  E[tokens](k) = (1 - a^(k+1)) / (1 - a) for a per-draft acceptance rate a
  (an exponential moving average of observed acceptance), over
  cost(k) = 1 + beta(load) * k, with hysteresis so k changes only when the
  gain exceeds a margin.

The scheduler caps every request's drafts at the chosen k for the step (the
MTP head still drafts its full depth; drafts beyond the cap are not verified).
The reference's policy (vllm_sm80/spec_decode/adaptive_k.py:34 AdaptiveKConfig,
:191 AdaptiveKPolicy) chooses from the same two ideas.
"""

from __future__ import annotations

from dataclasses import dataclass, field


def expected_tokens(k: int, a: float) -> float:
    """Tokens produced by one verify step with k drafts and per-draft acceptance a (bonus included)."""
    if a >= 1.0:
        return float(k + 1)
    return (1.0 - a ** (k + 1)) / (1.0 - a)


@dataclass
class AdaptiveKPolicy:
    k_max: int
    mode: str = "by_load"
    table: list[tuple[int, int]] = field(default_factory=list)  # (max running requests, k)
    ema: float = 0.9
    margin: float = 0.05
    compute_bound_tokens: int = 512  # batch tokens at which a step stops being weight-streaming bound
    accept_rate: float = 0.6
    k: int = -1

    def __post_init__(self):
        if not self.table:
            km = self.k_max
            self.table = [(8, km), (32, max(1, km - 1)), (128, max(1, km - 2)), (1 << 30, 1)]
        if self.k < 0:
            self.k = self.k_max

    def observe(self, proposed: int, accepted: int) -> None:
        if proposed > 0:
            self.accept_rate = self.ema * self.accept_rate + (1.0 - self.ema) * (accepted / proposed)

    def beta(self, running: int) -> float:
        """Relative cost of one more draft token per request: near 0 while the step's token count is far
        below the compute-bound point, 1 at and beyond it."""
        return min(1.0, running * (1 + self.k) / self.compute_bound_tokens)

    def choose(self, running: int) -> int:
        if self.mode == "by_load":
            for bound, k in self.table:
                if running <= bound:
                    self.k = min(k, self.k_max)
                    return self.k
            self.k = 1
            return self.k
        b = self.beta(running)

        def score(k):
            return expected_tokens(k, self.accept_rate) / (1.0 + b * k)

        best = max(range(self.k_max + 1), key=score)
        if best != self.k and score(best) > score(self.k) * (1.0 + self.margin):
            self.k = best
        return self.k
