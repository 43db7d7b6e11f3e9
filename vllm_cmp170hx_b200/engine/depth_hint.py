"""Verify width per decode step from each request's last verified round.

The table ``full=W1,W2,...;base=W1,W2,...`` (``VLLM_B200_DEPTH_HINT``; the reference's
``VLLM_DSPARK_DEPTH_HINT``, vllm_sm80/spec_decode/dspark_depth_hint.py:1-31) names two width lists
indexed by the number of requests the engine holds (running + waiting; the last entry repeats):

* ``full`` -- the width of a step whose every decoding request accepted all the drafts of its last
  verified round, or whose output is a tool call or JSON by the request's own fields (the chat
  endpoint sets ``SamplingParams.certain_output`` when tools are offered with ``tool_choice`` other
  than ``"none"``, or a JSON ``response_format`` is asked for);
* ``base`` -- every other step, and a request's first decoding step.

A decode batch verifies one width, so one request without a full round keeps the step at ``base``.
The width is capped by the step's adaptive draft count (``adaptive_k``), and the scheduler verifies at
most that many of each request's drafts.  An empty table changes nothing.
"""

from __future__ import annotations

from dataclasses import dataclass, field

JSON_FORMATS = frozenset({"json_object", "json_schema", "structural_tag"})


def certain_output(body: dict) -> bool:
    """A chat request whose output is a tool call or JSON by its own fields."""
    if body.get("tools") and body.get("tool_choice", "auto") != "none":
        return True
    fmt = body.get("response_format") or {}
    return isinstance(fmt, dict) and fmt.get("type") in JSON_FORMATS


@dataclass
class DepthHint:
    full: tuple[int, ...]
    base: tuple[int, ...]
    rounds: dict[str, bool] = field(default_factory=dict)  # request -> its last verified round was full

    @staticmethod
    def parse(raw: str) -> "DepthHint | None":
        raw = (raw or "").strip()
        if not raw:
            return None
        lists: dict[str, tuple[int, ...]] = {}
        for part in raw.split(";"):
            name, _, values = part.partition("=")
            name = name.strip()
            if name not in ("full", "base"):
                raise ValueError(f"depth hint: unknown list {name!r} (expected full= and base=)")
            try:
                lists[name] = tuple(int(v) for v in values.split(","))
            except ValueError as e:
                raise ValueError(f"depth hint: {name}= needs comma-separated integers, got {values!r}") from e
            if not lists[name] or min(lists[name]) < 0:
                raise ValueError(f"depth hint: {name}= needs non-negative widths")
        if set(lists) != {"full", "base"}:
            raise ValueError("depth hint needs both full= and base=")
        return DepthHint(lists["full"], lists["base"])

    def width(self, name: str, load: int) -> int:
        v = self.full if name == "full" else self.base
        return v[min(max(load, 1), len(v)) - 1]

    def observe(self, request_id: str, num_draft: int, num_accepted: int) -> None:
        """Record whether a verified round accepted every draft (rounds without drafts say nothing)."""
        if num_draft > 0:
            self.rounds[request_id] = num_accepted >= num_draft

    def forget(self, request_id: str) -> None:
        self.rounds.pop(request_id, None)

    def select(self, decoding: list, load: int, cap: int) -> int:
        """The step's verify width: ``full`` or ``base`` at this load, at most ``cap``."""
        full = bool(decoding) and all(self.rounds.get(r.request_id, False) or r.params.certain_output
                                      for r in decoding)
        return min(self.width("full" if full else "base", load), cap)
