"""Public engine API.

    engine = LLMEngine(EngineConfig(...))
    engine.add_request(prompt_token_ids, SamplingParams(max_tokens=...))
    while engine.has_unfinished():
        for out in engine.step(): ...

    LLM(cfg).generate(list_of_prompts, params) -> list[RequestOutput]

Multi-GPU (tensor parallel) runs SPMD: one process per GPU, every rank runs
the same scheduler on the same request stream (the API server broadcasts new
requests from rank 0 over the gloo group), so all ranks build identical
batches without a per-step metadata exchange; rank 0 returns outputs.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..config import EngineConfig
from ..parallel import state as pstate
from .request import Request, SamplingParams, Status
from .runner import ModelRunner
from .scheduler import Scheduler


# an output slot whose token is still on the device (asynchronous scheduling)
_PLACEHOLDER = -1


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: list[int]
    output_token_ids: list[int]
    finished: bool
    finish_reason: str | None = None
    new_token_ids: list[int] | None = None


class LLMEngine:
    def __init__(self, cfg: EngineConfig, model=None):
        self.cfg = cfg
        st = pstate.get()
        if st.tp_size != cfg.parallel.tensor_parallel_size:
            st = pstate.init(cfg.parallel.tensor_parallel_size, cfg.parallel.pipeline_parallel_size)
        st.expert_parallel = bool(cfg.parallel.expert_parallel)
        from .. import envs

        if not envs.get("VLLM_B200_CUDA_GRAPHS"):
            cfg.enforce_eager = True
        envs.log_gate("CUDA graphs for decode steps", not cfg.enforce_eager)
        self.runner = ModelRunner(cfg, model)
        self._setup_sequence_parallel(st)
        self.scheduler = Scheduler(cfg.scheduler, cfg.cache, self.runner.block_pool, self.runner.slot_pool)
        self._diagnostics(st)
        self.adaptive_k = None
        self._k_seen = (0, 0)
        mode = cfg.scheduler.adaptive_k or ""
        if not mode:
            from .. import envs

            mode = envs.get("VLLM_B200_ADAPTIVE_K")
        if mode and cfg.scheduler.num_speculative_tokens > 0:
            from .adaptive_k import AdaptiveKPolicy

            self.adaptive_k = AdaptiveKPolicy(cfg.scheduler.num_speculative_tokens,
                                              mode if mode in ("by_load", "accept") else "by_load")
        self.depth_hint = None
        if cfg.scheduler.num_speculative_tokens > 0:
            from .. import envs
            from .depth_hint import DepthHint

            self.depth_hint = DepthHint.parse(envs.get("VLLM_B200_DEPTH_HINT"))
        self.requests: dict[str, Request] = {}
        self.num_steps = 0
        self.k_hist: dict[int, int] = {}  # draft count chosen per step (adaptive k) -> steps
        self.eos_token_id: int | None = None

    def _setup_sequence_parallel(self, st) -> None:
        """Expert-parallel groups run steps in the sequence-parallel layout (parallel/sp.py) over
        torch.distributed until a fused transport replaces it (parallel/symm.py)."""
        from .. import envs
        from ..parallel import comm
        from ..parallel.sp import TorchSP

        comm.enable_sp(None)
        p = self.cfg.parallel
        model = self.runner.model
        mode = envs.get("VLLM_B200_EP_DISPATCH")
        if mode not in ("symm", "nccl", "off"):
            raise ValueError(f"VLLM_B200_EP_DISPATCH={mode!r}: 'symm', 'nccl' or 'off'")
        if (st.tp_size > 1 and not st.emulated and p.expert_parallel and p.sequence_parallel and mode != "off"
                and hasattr(model, "supports_sp") and model.supports_sp()):
            comm.enable_sp(TorchSP(st.tp_group, model.cfg.hidden_size, model.cfg.moe.top_k))

    def _diagnostics(self, st) -> None:
        from .. import envs
        from ..utils import memory
        from ..utils.capture import KernelCapture

        envs.check_environment()
        if envs.get("VLLM_B200_MEM_ATTRIBUTION"):
            memory.log_attribution(self.runner.model, st.rank)
        if envs.get("VLLM_B200_KV_PLAN_LOG"):
            memory.log_kv_plan(self.runner, st.rank)
        self.capture = KernelCapture.from_env(st.rank)
        if self.capture is not None:
            self.capture.install()
        envs.log_gate("kernel-call capture", self.capture is not None)
        from ..dev.ab import DevAB, HotSwap

        self.dev_ab = DevAB.from_env(self)
        self.hot_swap = HotSwap.from_env()
        if self.hot_swap is not None:
            self.hot_swap.swap_in()
        envs.log_gate("dev A/B switch", self.dev_ab is not None)
        envs.log_gate("hot swap", self.hot_swap is not None)

    def warmup(self, capture_graphs: bool = True) -> dict[int, int]:
        """Kernel warm-up (one throwaway prefill + decode) and, on the GPU, capture of every decode
        graph; returns the bytes each graph capture kept (logged).  Every rank calls it at start-up."""
        import logging

        self.runner.warmup()
        kept = self.runner.capture_graphs() if capture_graphs else {}
        if kept:
            tr = self.runner.graph_transient
            logging.getLogger("vllm_cmp170hx_b200").info(
                "CUDA graphs captured: %s", ", ".join(f"batch {b}: {v / 2**20:.1f} MiB kept, "
                                                      f"{tr.get(b, 0) / 2**20:.1f} MiB transient"
                                                      for b, v in kept.items()))
        return kept

    def profile(self, steps: int, out_dir: str) -> str:
        """Run `steps` engine steps under the torch profiler and write this rank's chrome trace
        (plus an execution trace with VLLM_B200_EXECUTION_TRACE; ranks export one after another with
        VLLM_B200_SERIAL_TRACE_EXPORT).  Returns the trace path."""
        import contextlib
        import os

        from torch.profiler import ProfilerActivity, profile as tprofile

        from .. import envs
        from ..utils import trace

        st = pstate.get()
        os.makedirs(out_dir, exist_ok=True)
        stem = os.path.join(out_dir, f"rank{st.rank}")
        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
        et = trace.execution_trace(stem) if envs.get("VLLM_B200_EXECUTION_TRACE") else contextlib.nullcontext()
        with et, tprofile(activities=acts) as prof:
            for _ in range(steps):
                if not self.has_unfinished():
                    break
                self.step()
            if torch.cuda.is_available():
                torch.cuda.synchronize()
        path = stem + ".trace.json"
        if envs.get("VLLM_B200_SERIAL_TRACE_EXPORT") and st.world_size > 1:
            trace.serial_export(prof, path, st.rank, st.world_size, out_dir)
        else:
            prof.export_chrome_trace(path)
        return path

    def add_request(self, prompt_token_ids: list[int], params: SamplingParams | None = None,
                    request_id: str | None = None, synthetic_prefix: int = 0) -> str:
        """synthetic_prefix (benchmarks): that many leading prompt positions are taken as already
        computed, their cache rows being whatever the caches hold (see ModelRunner.fill_caches_random)."""
        req = Request(list(prompt_token_ids), params or SamplingParams(), request_id or "",
                      eos_token_id=self.eos_token_id, synthetic_prefix=synthetic_prefix)
        self.scheduler.add(req)
        self.requests[req.request_id] = req
        return req.request_id

    def abort_request(self, request_id: str) -> None:
        self.scheduler.abort(request_id)
        self.requests.pop(request_id, None)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work() or self._inflight is not None

    _inflight = None  # asynchronous scheduling: (scheduler output, runner handle) of the step in flight

    def _async_on(self) -> bool:
        r = self.runner
        return (self.cfg.scheduler.async_scheduling and r.st.pp_size == 1 and r.spec is None
                and self.adaptive_k is None and not r._ngram_sources())

    def step(self) -> list[RequestOutput]:
        if self._inflight is not None or self._async_on():
            return self._step_async()
        return self._step_sync()

    # ------------------------------------------------------------------ asynchronous scheduling
    def _step_async(self) -> list[RequestOutput]:
        """Decode steps overlap the host: step N+1 is scheduled (its requests' step-N tokens taken as
        placeholders) and launched -- its input ids gathered on the device from step N's sampled tokens --
        before step N's tokens are read back and applied.  A request whose step-N token stops it has one
        extra position computed in step N+1, which is discarded.  Steps that need the host to know every
        token (admissions, prefill chunks, preemption victims coming back) run synchronously after the
        step in flight is drained (the reference's async scheduler, vllm_sm80/sched/scheduler.py:439-444,
        over upstream's placeholder scheduling)."""
        sch, r = self.scheduler, self.runner
        if self._inflight is None:
            out = sch.schedule()
            if not out.reqs:
                return []
            if not (self._async_on() and r.can_launch(out)):
                return self._execute_sync(out)
            self._inflight = (out, r.launch(out))
            self.num_steps += 1
            return []
        out_n, h_n = self._inflight
        self._inflight = None
        nxt = self._schedule_ahead(out_n) if (self._async_on() and not sch.waiting) else None
        h_next = r.launch(nxt, prev=(out_n, h_n)) if nxt is not None else None
        res = self._finalize(out_n, h_n)
        if h_next is not None:
            self._inflight = (nxt, h_next)
            self.num_steps += 1
        return res

    def _schedule_ahead(self, out_n):
        """Schedule the step after `out_n` (in flight) with its tokens as placeholders; None when that
        step could not be one launchable decode step."""
        sch, r = self.scheduler, self.runner
        live = [s for s in out_n.reqs if not s.req.status.finished]
        if not live or len(sch.running) > max(self.cfg.cuda_graph_batch_sizes) or any(
                s.num_new != 1 or not s.sample for s in live):
            return None
        for s in live:
            req = s.req
            req.output_token_ids.append(_PLACEHOLDER)
            req.num_computed_tokens = s.start + 1
            req.async_hold = (len(req.output_token_ids) >= req.params.max_tokens
                              or req.num_tokens >= self.cfg.scheduler.max_model_len)
        nxt = sch.schedule(admit=False)
        if not nxt.reqs or not r.can_launch(nxt):
            # nothing to run ahead: those requests are scheduled again after the drain, which fills their
            # placeholders (blocks grown for them stay theirs)
            return None
        return nxt

    def _finalize(self, out_n, h_n) -> list[RequestOutput]:
        """Read back a launched step's tokens, put them in place of the placeholders (or append them),
        check stops and retire finished requests; returns that step's outputs."""
        from .failed_inputs import FAILED_TOKEN

        sch = self.scheduler
        sampled = self.runner.finish(out_n, h_n)
        now = time.monotonic()
        done, res = [], []
        for s in out_n.reqs:
            req = s.req
            if req.status.finished:
                continue  # stopped by its previous token: this step's position is discarded
            toks = sampled.get(req.request_id, [])
            i = s.start + 1 - req.num_prompt_tokens  # output index of this step's token
            ahead = i < len(req.output_token_ids) and req.output_token_ids[i] == _PLACEHOLDER
            req.async_hold = False
            if not toks or FAILED_TOKEN in toks:
                if ahead:
                    del req.output_token_ids[i:]
                req.status = Status.FINISHED_ERROR
                done.append(req)
            else:
                if ahead:
                    req.output_token_ids[i] = int(toks[0])
                else:
                    req.num_computed_tokens = s.start + 1
                    req.output_token_ids.append(int(toks[0]))
                if req.first_token_time is None:
                    req.first_token_time = now
                req.token_times.append(now)
                if req.check_stop():
                    done.append(req)
            res.append(RequestOutput(req.request_id, req.prompt_token_ids, list(req.output_token_ids),
                                     req.status.finished,
                                     req.status.value.replace("finished_", "") if req.status.finished else None,
                                     [] if req.status == Status.FINISHED_ERROR else [req.output_token_ids[-1]]))
        for req in done:
            if req in sch.running:
                sch.running.remove(req)
            elif req in sch.waiting:  # preempted while scheduling ahead
                sch.waiting.remove(req)
            sch._release(req)
            sch.finished.append(req)
            self.requests.pop(req.request_id, None)
        return res

    # ------------------------------------------------------------------ synchronous steps
    def _step_sync(self) -> list[RequestOutput]:
        if self.adaptive_k is not None:
            spec = self.runner.spec
            if spec is not None:
                st = spec.stats
                self.adaptive_k.observe(st["proposed"] - self._k_seen[0], st["accepted"] - self._k_seen[1])
                self._k_seen = (st["proposed"], st["accepted"])
            self.scheduler.draft_cap = self.adaptive_k.choose(len(self.scheduler.running))
            k = self.scheduler.draft_cap
            self.k_hist[k] = self.k_hist.get(k, 0) + 1
        if self.depth_hint is not None:
            sch = self.scheduler
            cap = sch.draft_cap if self.adaptive_k is not None else self.cfg.scheduler.num_speculative_tokens
            decoding = [r for r in sch.running if r.num_computed_tokens == r.num_tokens - 1]
            sch.draft_cap = self.depth_hint.select(decoding, len(sch.running) + len(sch.waiting), cap)
        self._host_width()
        out = self.scheduler.schedule()
        if not out.reqs:
            return []
        return self._execute_sync(out)

    def _host_width(self) -> None:
        """The depth policy's host width: a decode-only step of b requests (b in its batch sizes)
        verifies the K its objective picks from each request's p_i of an earlier round."""
        spec = self.runner.spec
        hw = getattr(getattr(spec, "depth", None), "host_width", None) if spec is not None else None
        if hw is None:
            return
        sch = self.scheduler
        decoding = [r for r in sch.running if r.num_computed_tokens == r.num_tokens - 1]
        if not decoding or len(decoding) != len(sch.running) or sch.waiting:
            return  # steps with prefill rows keep the width the load gave
        cap = (sch.draft_cap if (self.adaptive_k is not None or self.depth_hint is not None)
               else self.cfg.scheduler.num_speculative_tokens)
        K = hw.choose([spec.p_round(r.request_id, hw.lag) for r in decoding], len(decoding), cap)
        sch.draft_cap = cap if K is None else K

    def _execute_sync(self, out) -> list[RequestOutput]:
        before = {s.req.request_id: len(s.req.output_token_ids) for s in out.reqs}
        sampled = self.runner.execute(out)
        if self.depth_hint is not None:
            for s in out.reqs:
                if s.num_draft:
                    self.depth_hint.observe(s.req.request_id, s.num_draft,
                                            max(0, len(sampled.get(s.req.request_id, [])) - 1))
        self.scheduler.update(out, sampled)
        self.runner.propose()
        self.num_steps += 1
        res = []
        for s in out.reqs:
            r = s.req
            new = r.output_token_ids[before[r.request_id]:]
            if new or r.status.finished:
                res.append(RequestOutput(r.request_id, r.prompt_token_ids, list(r.output_token_ids),
                                         r.status.finished,
                                         r.status.value.replace("finished_", "") if r.status.finished else None, new))
            if r.status.finished:
                self.requests.pop(r.request_id, None)
                if self.depth_hint is not None:
                    self.depth_hint.forget(r.request_id)
                if self.runner.spec is not None:
                    self.runner.spec.p_rounds.pop(r.request_id, None)
        return res


def metrics_lines(engine: "LLMEngine") -> list[str]:
    """Prometheus text lines of the engine's counters: steps, speculative decoding (drafts proposed /
    accepted, acceptance rate, drafts the verify-depth policy cut), the adaptive draft count chosen per
    step as a histogram, and the last step's device time."""
    lines = [f"b200_engine_steps_total {engine.num_steps}"]
    spec = getattr(engine.runner, "spec", None)
    if spec is not None:
        st = spec.stats
        lines += [f"b200_spec_draft_tokens_total {st['proposed']}", f"b200_spec_accepted_tokens_total {st['accepted']}",
                  f"b200_spec_acceptance_rate {spec.acceptance_rate():.6f}",
                  f"b200_spec_depth_cut_tokens_total {st.get('depth_cut', 0)}",
                  f'b200_spec_method{{method="{spec.method}"}} 1']
    for k in sorted(engine.k_hist):
        lines.append(f'b200_adaptive_k_steps{{k="{k}"}} {engine.k_hist[k]}')
    last = getattr(engine.runner, "last_stats", None)
    if last is not None and getattr(last, "device_ms", None):
        lines.append(f"b200_last_step_device_ms {last.device_ms:.4f}")
    return lines


class LLM:
    """Offline batch generation over :class:`LLMEngine`."""

    def __init__(self, cfg: EngineConfig, model=None):
        self.engine = LLMEngine(cfg, model)

    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None
                 ) -> list[RequestOutput]:
        if not isinstance(params, list):
            params = [params or SamplingParams()] * len(prompts)
        ids = [self.engine.add_request(p, sp) for p, sp in zip(prompts, params)]
        done: dict[str, RequestOutput] = {}
        while self.engine.has_unfinished():
            for o in self.engine.step():
                if o.finished:
                    done[o.request_id] = o
        return [done[i] for i in ids]
