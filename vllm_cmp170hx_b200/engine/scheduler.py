"""Continuous-batching scheduler with chunked prefill.

Each step gets a token budget (`max_num_batched_tokens`).  Running requests
are served first: a decoding request takes 1 token (plus its draft tokens
under speculative decoding), a request still in prefill takes the next chunk
of its prompt.  Waiting requests are admitted while budget, sequence slots,
KV blocks and recurrent-state slots last.  A request that cannot grow its KV
is handled by preempting the most recently admitted running request
(recompute: its blocks and state slot are freed and it re-enters the queue
head with `num_computed_tokens = 0`).

Fair chunked prefill (the reference's `--prefill-chunk-with-decodes`,
`--max-num-partial-prefills`, vllm_sm80/sched/step.py:36 Sm80Step): at most
`max_num_partial_prefills` requests are in a partial prefill at once and a
request's chunk is capped at `long_prefill_token_threshold` when set.  With
`prefill_chunk_with_decodes` > 0 and some running request decoding, prefill
chunks also draw on a second, prefill-only budget of that many tokens, split
evenly between the prompts that can advance this step (running chunks and
admissible waiting prompts, up to `max_num_partial_prefills`); decode tokens
never draw on it, so decodes keep their slot in every step while long prompts
are chunked.  Prompts the short-prompt bypass exempts are neither capped nor
charged.  (Requests are preempted only from the back of the running list,
after the ones already scheduled this step, so no charge needs a refund.)
"""

from __future__ import annotations

import collections
import time
from dataclasses import dataclass, field

from ..config import CacheConfig, SchedulerConfig
from .failed_inputs import FAILED_TOKEN
from .request import Request, Status


@dataclass
class ScheduledReq:
    req: Request
    num_new: int  # tokens computed this step
    start: int  # first position computed this step
    sample: bool  # the step ends at the request's last known token -> sample
    num_draft: int = 0


@dataclass
class SchedulerOutput:
    reqs: list[ScheduledReq] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return sum(s.num_new for s in self.reqs)

    @property
    def decode_only(self) -> bool:
        return bool(self.reqs) and all(s.num_new == 1 + s.num_draft and s.start > 0 for s in self.reqs)


def block_hashes(tokens: list[int], block_size: int) -> list[int]:
    """Chained hashes of the full blocks of `tokens`: block i's hash covers every token up to its end,
    so equal hashes mean equal prefixes (ints only: the same on every rank and every run)."""
    out, h = [], 0x9E3779B97F4A7C15
    for i in range(len(tokens) // block_size):
        h = hash((h, tuple(tokens[i * block_size:(i + 1) * block_size]))) & 0x7FFFFFFFFFFFFFFF
        out.append(h)
    return out


class Scheduler:
    def __init__(self, sched: SchedulerConfig, cache: CacheConfig, block_pool, slot_pool=None):
        self.cfg = sched
        self.block_size = cache.block_size
        self.blocks = block_pool
        self.slots = slot_pool
        # Prefix caching: a full block of computed prompt tokens is registered under its chained hash
        # once the step that computed it succeeded; a later request whose prompt starts with the same
        # blocks takes them (reference counted) and starts computing after them.  Models with
        # recurrent state (KDA / DeepSeek-V4.1 rings) keep no per-block state, so it is off for them.
        self.prefix_caching = bool(cache.enable_prefix_caching) and slot_pool is None
        self.prefix_hits = 0  # tokens taken from the cache (metrics)
        self.waiting: collections.deque[Request] = collections.deque()
        self.running: list[Request] = []
        self.finished: list[Request] = []
        # speculative decoding: KV blocks reserved past a sampling step for the drafter's own cache writes
        self.lookahead = max(0, sched.num_speculative_tokens - 1)
        from .. import envs

        # prompts up to this length are never held back by the partial-prefill cap (the reference's
        # VLLM_FAIR_PREFILL_SHORT_BYPASS): they finish in one chunk and cost the decodes little
        self.short_bypass = envs.get("VLLM_B200_FAIR_PREFILL_SHORT_BYPASS")
        self.draft_cap = sched.num_speculative_tokens  # drafts verified per request this step (adaptive k)

    # ------------------------------------------------------------------ API
    def add(self, req: Request) -> None:
        if req.num_prompt_tokens + req.params.max_tokens > self.cfg.max_model_len:
            req.params.max_tokens = max(1, self.cfg.max_model_len - req.num_prompt_tokens)
        if req.num_prompt_tokens >= self.cfg.max_model_len:
            raise ValueError(f"prompt of {req.num_prompt_tokens} tokens exceeds max_model_len {self.cfg.max_model_len}")
        req.arrival = req.arrival or time.monotonic()
        self.waiting.append(req)

    def abort(self, request_id: str) -> bool:
        for q in (self.running, self.waiting):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    r.status = Status.FINISHED_ABORTED
                    self._release(r)
                    return True
        return False

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ------------------------------------------------------------------ helpers
    def _blocks_needed(self, req: Request, upto: int) -> int:
        need = (upto + self.block_size - 1) // self.block_size
        return max(0, need - len(req.block_ids))

    def _grow(self, req: Request, upto: int) -> bool:
        n = self._blocks_needed(req, upto)
        if n == 0:
            return True
        if self.blocks.num_free() < n:
            return False
        req.block_ids.extend(int(b) for b in self.blocks.allocate(n))
        return True

    def _release(self, req: Request) -> None:
        if req.block_ids:
            self.blocks.free(req.block_ids)  # registered blocks stay findable until reallocated (LRU)
            req.block_ids = []
        req.num_cached_blocks = 0
        if self.slots is not None and req.kda_slot > 0:
            self.slots.free(req.kda_slot)
        req.kda_slot = -1

    def _take_cached_prefix(self, req: Request) -> None:
        """Reuse the longest run of cached leading blocks of the prompt (at least the last prompt token
        is always computed, it is sampled from)."""
        if not req.block_hashes:
            req.block_hashes = block_hashes(req.prompt_token_ids, self.block_size)
        hits = []
        usable = (req.num_prompt_tokens - 1) // self.block_size
        for h in req.block_hashes[:usable]:
            b = int(self.blocks.lookup(h))
            if b < 0:
                break
            hits.append(b)
        for b in hits:
            self.blocks.touch(b)
        req.block_ids = hits
        req.num_cached_blocks = len(hits)
        req.num_computed_tokens = len(hits) * self.block_size
        req.num_prefix_hit_tokens = req.num_computed_tokens
        self.prefix_hits += req.num_computed_tokens

    def _register_blocks(self, req: Request) -> None:
        """Register the prompt blocks this request has fully computed under their hashes."""
        if not req.block_hashes:
            req.block_hashes = block_hashes(req.prompt_token_ids, self.block_size)
        full = min(req.num_computed_tokens // self.block_size, len(req.block_hashes), len(req.block_ids))
        for j in range(req.num_cached_blocks, full):
            self.blocks.cache_block(req.block_ids[j], req.block_hashes[j])
        req.num_cached_blocks = max(req.num_cached_blocks, full)

    def _preempt(self, victim: Request, out: SchedulerOutput) -> None:
        self.running.remove(victim)
        self._release(victim)
        victim.num_computed_tokens = 0
        victim.num_preemptions += 1
        victim.status = Status.PREEMPTED
        victim.draft_token_ids = []
        victim.draft_live = -1
        self.waiting.appendleft(victim)
        out.preempted.append(victim)

    # ------------------------------------------------------------------ schedule
    def _prefill_budget(self, budget: int) -> tuple[int, int]:
        """This step's prefill-only budget and per-prompt chunk cap (both = budget when off or when no
        running request decodes)."""
        total = budget
        if self.cfg.prefill_chunk_with_decodes > 0 and any(
                r.num_tokens - r.num_computed_tokens <= 1 and r.num_computed_tokens > 0 for r in self.running):
            total = min(total, self.cfg.prefill_chunk_with_decodes)
        per = total
        if self.cfg.prefill_chunk_with_decodes > 0 and self.cfg.max_num_partial_prefills > 0:
            n = sum(1 for r in self.running
                    if (r.num_tokens - r.num_computed_tokens > 1 or r.num_computed_tokens == 0)
                    and r.num_prompt_tokens > self.short_bypass)
            n += sum(1 for r in list(self.waiting)[: self.cfg.max_num_partial_prefills]
                     if r.num_prompt_tokens > self.short_bypass)
            n = min(max(n, 1), self.cfg.max_num_partial_prefills)
            per = max(1, total // n)
        return total, per

    def schedule(self, admit: bool = True) -> SchedulerOutput:
        """One step's work.  admit=False schedules only running requests (asynchronous scheduling ahead
        of a step in flight, whose tokens are not known on the host yet)."""
        out = SchedulerOutput()
        budget = self.cfg.max_num_batched_tokens
        partial = 0
        cap = self.cfg.long_prefill_token_threshold or budget
        prefill_left, per_prompt = self._prefill_budget(budget)
        scheduled_ids = set()
        i = 0
        while i < len(self.running):
            req = self.running[i]
            if req.async_hold:
                i += 1
                continue
            remaining = req.num_tokens - req.num_computed_tokens
            if remaining > 1 or (req.num_computed_tokens == 0):
                # still in prefill (the last prompt token is computed together with sampling)
                if partial >= self.cfg.max_num_partial_prefills and req.num_prompt_tokens > self.short_bypass:
                    i += 1
                    continue
                n = min(remaining, budget, cap)
                if req.num_prompt_tokens > self.short_bypass:
                    n = min(n, per_prompt, prefill_left)
                drafts = 0
            else:
                drafts = min(len(req.draft_token_ids), max(0, budget - 1), self.draft_cap)
                n = 1 + drafts
            if n <= 0 or n > budget:
                i += 1
                continue
            upto = req.num_computed_tokens + n
            if upto >= req.num_tokens:
                # the drafter writes its cache up to k-1 positions past this step
                upto = min(upto + self.lookahead, self.cfg.max_model_len)
            while not self._grow(req, upto):
                victim = self.running[-1]
                if victim is req:
                    break
                self._preempt(victim, out)
            if self._blocks_needed(req, upto) > 0:
                # could not make room even alone: preempt this one
                self._preempt(req, out)
                continue
            sample = req.num_computed_tokens + n >= req.num_tokens
            if not sample:
                partial += 1
            if drafts == 0 and n > 1 and req.num_prompt_tokens > self.short_bypass:
                prefill_left -= n
            out.reqs.append(ScheduledReq(req, n, req.num_computed_tokens, sample, drafts))
            scheduled_ids.add(req.request_id)
            budget -= n
            i += 1
        # admit waiting requests
        while admit and self.waiting and budget > 0 and len(self.running) < self.cfg.max_num_seqs:
            req = self.waiting[0]
            if (partial >= self.cfg.max_num_partial_prefills and req.num_tokens > budget
                    and req.num_prompt_tokens > self.short_bypass):
                break
            if req.synthetic_prefix and req.num_computed_tokens == 0:
                req.num_computed_tokens = min(req.synthetic_prefix, req.num_prompt_tokens - 1)
            elif self.prefix_caching and req.num_computed_tokens == 0 and not req.block_ids:
                self._take_cached_prefix(req)
            n = min(req.num_tokens - req.num_computed_tokens, budget, cap)
            charged = req.num_tokens - req.num_computed_tokens > 1 and req.num_prompt_tokens > self.short_bypass
            if charged:
                if prefill_left <= 0:
                    break
                n = min(n, per_prompt, prefill_left)
            upto = req.num_computed_tokens + n
            if upto >= req.num_tokens:
                upto = min(upto + self.lookahead, self.cfg.max_model_len)
            if self._blocks_needed(req, upto) > self.blocks.num_free():
                break
            if self.slots is not None and req.kda_slot <= 0 and self.slots.num_free() == 0:
                break
            self.waiting.popleft()
            if self.slots is not None and req.kda_slot <= 0:
                req.kda_slot = self.slots.allocate()
            self._grow(req, upto)
            req.status = Status.RUNNING
            self.running.append(req)
            sample = req.num_computed_tokens + n >= req.num_tokens
            if not sample:
                partial += 1
            if charged:
                prefill_left -= n
            out.reqs.append(ScheduledReq(req, n, req.num_computed_tokens, sample, 0))
            budget -= n
        return out

    # ------------------------------------------------------------------ update
    def update(self, out: SchedulerOutput, sampled: dict[str, list[int]]) -> list[Request]:
        """Advance computed counts, append sampled tokens (accepted drafts + the
        bonus token under speculative decoding) and retire finished requests."""
        now = time.monotonic()
        done = []
        for s in out.reqs:
            req = s.req
            if req.status.finished:
                continue
            toks = sampled.get(req.request_id, [])
            if FAILED_TOKEN in toks:
                # no valid token from this step (poisoned inputs): finish with an error, drop the step;
                # the blocks it computed are never registered for prefix reuse
                req.status = Status.FINISHED_ERROR
                req.draft_token_ids = []
                req.draft_live = -1
                done.append(req)
                continue
            if s.num_draft:
                # verify step: positions of rejected drafts are recomputed later
                accepted = max(0, len(toks) - 1)
                req.num_computed_tokens = s.start + 1 + accepted
            else:
                req.num_computed_tokens = s.start + s.num_new
            if self.prefix_caching:
                self._register_blocks(req)
            req.draft_token_ids = []
            req.draft_live = -1
            for t in toks:
                req.output_token_ids.append(int(t))
                if req.first_token_time is None:
                    req.first_token_time = now
                req.token_times.append(now)
                if req.check_stop():
                    break
            if req.status.finished:
                done.append(req)
        for req in done:
            if req in self.running:
                self.running.remove(req)
            self._release(req)
            self.finished.append(req)
        return done
