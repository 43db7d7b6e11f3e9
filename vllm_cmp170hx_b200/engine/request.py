"""Request lifecycle state and sampling parameters."""

from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0  # 0: greedy
    top_p: float = 1.0
    top_k: int = 0
    stop_token_ids: list[int] = field(default_factory=list)
    ignore_eos: bool = False
    seed: int | None = None
    # tokens that are never sampled (at most 4; e.g. a parser's tool-call opener under tool_choice="none")
    bad_token_ids: list[int] = field(default_factory=list)
    # the output is a tool call or JSON by the request's own fields (a verify-width hint; chat endpoint)
    certain_output: bool = False


class Status(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED_STOPPED = "finished_stopped"
    FINISHED_LENGTH = "finished_length"
    FINISHED_ABORTED = "finished_aborted"
    FINISHED_ERROR = "finished_error"

    @property
    def finished(self) -> bool:
        return self in _FINISHED


_FINISHED = frozenset(s for s in Status if s.value.startswith("finished"))


_ids = itertools.count()


@dataclass
class Request:
    prompt_token_ids: list[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    request_id: str = ""
    eos_token_id: int | None = None
    arrival: float = 0.0
    status: Status = Status.WAITING
    output_token_ids: list[int] = field(default_factory=list)
    num_computed_tokens: int = 0
    block_ids: list[int] = field(default_factory=list)
    kda_slot: int = -1
    num_preemptions: int = 0
    first_token_time: float | None = None
    token_times: list[float] = field(default_factory=list)
    # speculative decoding: draft tokens proposed for the next verify step, and how many of them are live
    # (the verify-depth policy's row mask: drafts past it are verified rows whose results are ignored,
    # so every request keeps the same verify width; -1 = all live)
    draft_token_ids: list[int] = field(default_factory=list)
    draft_live: int = -1
    # benchmarks: the first `synthetic_prefix` prompt positions count as computed on admission (their
    # cache rows and recurrent state are whatever the caches hold, e.g. random rows), so a long-context
    # decode can be measured without prefilling it
    synthetic_prefix: int = 0
    # prefix caching: hashes of the prompt's full blocks (chained) and how many of this request's blocks
    # are registered in the block pool's hash table
    block_hashes: list[int] = field(default_factory=list)
    num_cached_blocks: int = 0
    num_prefix_hit_tokens: int = 0
    # asynchronous scheduling: the request ends with the step in flight whatever its token (length
    # limit), so the step scheduled ahead leaves it out
    async_hold: bool = False

    def __post_init__(self):
        if not self.request_id:
            self.request_id = f"req-{next(_ids)}"

    @property
    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    def token_at(self, i: int) -> int:
        """Token i of prompt + output without building the concatenation."""
        n = len(self.prompt_token_ids)
        return self.prompt_token_ids[i] if i < n else self.output_token_ids[i - n]

    def tokens(self, a: int, b: int) -> list[int]:
        """Tokens [a, b) of prompt + output without building the whole concatenation."""
        n = len(self.prompt_token_ids)
        if b <= n:
            return self.prompt_token_ids[a:b]
        if a >= n:
            return self.output_token_ids[a - n:b - n]
        return self.prompt_token_ids[a:] + self.output_token_ids[:b - n]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def in_prefill(self) -> bool:
        return self.num_computed_tokens < self.num_tokens - 1

    def check_stop(self) -> bool:
        if len(self.output_token_ids) >= self.params.max_tokens:
            self.status = Status.FINISHED_LENGTH
            return True
        if self.output_token_ids:
            last = self.output_token_ids[-1]
            if not self.params.ignore_eos and self.eos_token_id is not None and last == self.eos_token_id:
                self.status = Status.FINISHED_STOPPED
                return True
            if last in self.params.stop_token_ids:
                self.status = Status.FINISHED_STOPPED
                return True
        return False
