"""SPMD driving of a multi-rank engine: rank 0 owns the request stream; each
iteration it broadcasts a control message (new requests, aborts, stop) over
the CPU (gloo) group, then every rank applies it and runs the same step.
All ranks therefore build identical batches with no per-step tensor
metadata exchange (the reference relies on upstream vLLM's executor to
ship SchedulerOutput to every worker; here the scheduler is replicated)."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch.distributed as dist

from ..parallel import state as pstate
from .llm_engine import LLMEngine, RequestOutput
from .request import SamplingParams


@dataclass
class Control:
    new: list[tuple[str, list[int], SamplingParams]] = field(default_factory=list)
    aborts: list[str] = field(default_factory=list)
    stop: bool = False
    ab_flip: bool = False  # flip the dev A/B switch before this step (every rank at the same step)


class SPMDEngine:
    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self.st = pstate.get()

    def _exchange(self, ctl: Control | None) -> Control:
        if self.st.world_size == 1:
            return ctl or Control()
        obj = [ctl if self.st.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=self.st.world_cpu_group)
        return obj[0]

    def step(self, ctl: Control | None = None) -> list[RequestOutput]:
        """Rank 0: pass the control message; followers call follow() instead."""
        ctl = self._exchange(ctl)
        for rid, prompt, params in ctl.new:
            self.engine.add_request(prompt, params, rid)
        for rid in ctl.aborts:
            self.engine.abort_request(rid)
        if ctl.ab_flip and self.engine.dev_ab is not None:
            self.engine.dev_ab.flip()
        if ctl.stop:
            return []
        return self.engine.step() if self.engine.has_unfinished() else []

    def follow(self) -> None:
        while True:
            ctl = self._exchange(None)
            for rid, prompt, params in ctl.new:
                self.engine.add_request(prompt, params, rid)
            for rid in ctl.aborts:
                self.engine.abort_request(rid)
            if ctl.ab_flip and self.engine.dev_ab is not None:
                self.engine.dev_ab.flip()
            if ctl.stop:
                return
            if self.engine.has_unfinished():
                self.engine.step()
