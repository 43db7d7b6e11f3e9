"""OpenAI-compatible (and Anthropic ``/v1/messages``) HTTP server.

    python -m vllm_cmp170hx_b200.api.server --model config3 --tp 1 --port 8000
    torchrun --nproc-per-node 4 -m vllm_cmp170hx_b200.api.server --model DIR --tp 4

Endpoints: /health, /v1/models, /v1/completions, /v1/chat/completions
(streaming SSE, reasoning and tool-call parsing), /v1/messages, /metrics
(Prometheus).  The engine runs in one background thread per process
(rank 0 serves HTTP and broadcasts each step's new requests; other ranks
follow, see engine/spmd.py).  Random-init weights are used when the model
is a preset name; a checkpoint directory uses its config.json.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import queue
import threading
import time
import uuid

try:  # at module level: handler annotations are resolved against module globals
    from fastapi import Request
except ImportError:  # pragma: no cover
    Request = object

from ..config import CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig
from ..engine.depth_hint import certain_output
from ..engine.llm_engine import LLMEngine
from ..engine.request import SamplingParams
from ..engine.spmd import Control, SPMDEngine
from . import parsers
from .tokenizer import get_tokenizer


class AsyncEngine:
    """Thread-safe front of the engine for asyncio handlers."""

    def __init__(self, spmd: SPMDEngine):
        self.spmd = spmd
        self.inbox: queue.Queue = queue.Queue()
        self.streams: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Queue]] = {}
        self.stats = {"requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "ttft": [], "tpot": []}
        self._stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def _loop(self):
        eng = self.spmd.engine
        while not self._stop:
            ctl = Control()
            try:
                while True:
                    item = self.inbox.get_nowait()
                    if item[0] == "add":
                        ctl.new.append(item[1:])
                    else:
                        ctl.aborts.append(item[1])
            except queue.Empty:
                pass
            if not ctl.new and not ctl.aborts and not eng.has_unfinished():
                time.sleep(0.002)
                if self.spmd.st.world_size > 1:
                    self.spmd.step(Control())  # keep followers in lock step
                continue
            for out in self.spmd.step(ctl):
                target = self.streams.get(out.request_id)
                self.stats["generated_tokens"] += len(out.new_token_ids or [])
                if target is not None:
                    loop, q = target
                    loop.call_soon_threadsafe(q.put_nowait, out)

    async def generate(self, prompt_ids: list[int], params: SamplingParams):
        rid = "req-" + uuid.uuid4().hex
        q: asyncio.Queue = asyncio.Queue()
        self.streams[rid] = (asyncio.get_running_loop(), q)
        self.stats["requests"] += 1
        self.stats["prompt_tokens"] += len(prompt_ids)
        self.inbox.put(("add", rid, prompt_ids, params))
        t0 = time.monotonic()
        first = None
        try:
            while True:
                out = await q.get()
                if first is None and out.new_token_ids:
                    first = time.monotonic()
                    self.stats["ttft"].append(first - t0)
                yield out
                if out.finished:
                    n = len(out.output_token_ids)
                    if first is not None and n > 1:
                        self.stats["tpot"].append((time.monotonic() - first) / (n - 1))
                    return
        finally:
            self.streams.pop(rid, None)

    def abort(self, rid: str):
        self.inbox.put(("abort", rid))

    def shutdown(self):
        self._stop = True


def _params(body: dict, default_max: int = 16) -> SamplingParams:
    stop_ids = body.get("stop_token_ids") or []
    return SamplingParams(max_tokens=int(body.get("max_tokens") or body.get("max_completion_tokens") or default_max),
                          temperature=float(body.get("temperature", 0.0) or 0.0),
                          top_p=float(body.get("top_p", 1.0) or 1.0), top_k=int(body.get("top_k", 0) or 0),
                          stop_token_ids=list(stop_ids), ignore_eos=bool(body.get("ignore_eos", False)),
                          seed=body.get("seed"))


def _think_open_in_prompt(tokenizer, ids: list[int]) -> bool:
    """Whether the chat template opened the reasoning block at the end of the prompt."""
    try:
        return tokenizer.decode(ids[-4:]).rstrip().endswith(parsers.THINK_OPEN)
    except Exception:  # noqa: BLE001 - a tokenizer without decode of special tokens
        return False


def build_app(engine: AsyncEngine, tokenizer, model_name: str, parser: str | None = None):
    """The HTTP app.  ``parser`` names the reasoning / tool-call markup of the served model
    (``api/parsers.PARSERS``: generic, glm45, glm47, ling3, deepseek_v41)."""
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="vllm_cmp170hx_b200")
    family = parsers.get_family(parser)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "vllm_cmp170hx_b200"}]}

    @app.get("/metrics")
    async def metrics():
        s = engine.stats
        lines = [f"b200_requests_total {s['requests']}", f"b200_prompt_tokens_total {s['prompt_tokens']}",
                 f"b200_generation_tokens_total {s['generated_tokens']}"]
        for name, vals in (("ttft_seconds", s["ttft"]), ("tpot_seconds", s["tpot"])):
            if vals:
                v = sorted(vals)
                lines.append(f'b200_{name}{{quantile="0.5"}} {v[len(v) // 2]}')
                lines.append(f"b200_{name}_count {len(v)}")
        from ..engine.llm_engine import metrics_lines

        lines += metrics_lines(engine.spmd.engine)
        return PlainTextResponse("\n".join(lines) + "\n")

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        prompt = body.get("prompt", "")
        ids = prompt if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt) else \
            tokenizer.encode(prompt if isinstance(prompt, str) else prompt[0])
        params = _params(body)
        cid = "cmpl-" + uuid.uuid4().hex[:24]
        if body.get("stream"):
            async def gen():
                async for out in engine.generate(ids, params):
                    chunk = {"id": cid, "object": "text_completion", "model": model_name,
                             "choices": [{"index": 0, "text": tokenizer.decode(out.new_token_ids or []),
                                          "finish_reason": out.finish_reason}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        last = None
        async for out in engine.generate(ids, params):
            last = out
        text = tokenizer.decode(last.output_token_ids)
        return JSONResponse({"id": cid, "object": "text_completion", "model": model_name,
                             "choices": [{"index": 0, "text": text, "finish_reason": last.finish_reason,
                                          "token_ids": last.output_token_ids}],
                             "usage": {"prompt_tokens": len(ids), "completion_tokens": len(last.output_token_ids),
                                       "total_tokens": len(ids) + len(last.output_token_ids)}})

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        messages = body.get("messages", [])
        ids = tokenizer.apply_chat_template(messages)
        params = _params(body)
        params.bad_token_ids = parsers.tool_choice_none_bans(family, body, tokenizer)
        params.certain_output = certain_output(body)
        tools, tool_choice = body.get("tools"), body.get("tool_choice", "auto")
        think_open = _think_open_in_prompt(tokenizer, ids)
        cid = "chatcmpl-" + uuid.uuid4().hex[:24]
        if body.get("stream"):
            async def gen():
                sp = parsers.StreamParser(family, tools, tool_choice, think_open_in_prompt=think_open)
                ncalls = 0
                async for out in engine.generate(ids, params):
                    r, c, calls = sp.feed(tokenizer.decode(out.new_token_ids or []))
                    if out.finished:
                        r2, c2, calls2 = sp.finish()
                        r, c, calls = r + r2, c + c2, calls + calls2
                    delta = {}
                    if r:
                        delta["reasoning_content"] = r
                    if c:
                        delta["content"] = c
                    if calls:  # each call goes out whole, in the chunk where its closer arrived
                        delta["tool_calls"] = [dict(t.to_openai(), index=ncalls + i) for i, t in enumerate(calls)]
                        ncalls += len(calls)
                    fin = ("tool_calls" if sp.calls else out.finish_reason) if out.finished else None
                    chunk = {"id": cid, "object": "chat.completion.chunk", "model": model_name,
                             "choices": [{"index": 0, "delta": delta, "finish_reason": fin}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        last = None
        async for out in engine.generate(ids, params):
            last = out
        text = tokenizer.decode(last.output_token_ids)
        p = parsers.parse(text, family, tools, tool_choice, think_open_in_prompt=think_open)
        msg = {"role": "assistant", "content": p.content or None}
        if p.reasoning:
            msg["reasoning_content"] = p.reasoning
        if p.calls:
            msg["tool_calls"] = [c.to_openai() for c in p.calls]
        return JSONResponse({"id": cid, "object": "chat.completion", "model": model_name,
                             "choices": [{"index": 0, "message": msg,
                                          "finish_reason": "tool_calls" if p.calls else last.finish_reason}],
                             "usage": {"prompt_tokens": len(ids), "completion_tokens": len(last.output_token_ids),
                                       "total_tokens": len(ids) + len(last.output_token_ids)}})

    @app.post("/v1/messages")
    async def messages(req: Request):
        body = await req.json()
        msgs = list(body.get("messages", []))
        if body.get("system"):
            msgs = [{"role": "system", "content": body["system"]}] + msgs
        ids = tokenizer.apply_chat_template(msgs)
        params = _params(body)
        last = None
        async for out in engine.generate(ids, params):
            last = out
        text = tokenizer.decode(last.output_token_ids)
        _, content = parsers.split_reasoning(text)
        return JSONResponse({"id": "msg_" + uuid.uuid4().hex[:24], "type": "message", "role": "assistant",
                             "model": model_name, "content": [{"type": "text", "text": content}],
                             "stop_reason": "max_tokens" if last.finish_reason == "length" else "end_turn",
                             "usage": {"input_tokens": len(ids), "output_tokens": len(last.output_token_ids)}})

    return app


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--prefill-chunk-with-decodes", type=int, default=0,
                    help="fair chunked prefill: the prefill-only token budget of a step while requests decode "
                         "(0: off)")
    ap.add_argument("--max-num-partial-prefills", type=int, default=1)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--pp", type=int, default=1, help="pipeline-parallel stages")
    ap.add_argument("--enable-expert-parallel", action="store_true", help="routed experts split whole over TP")
    ap.add_argument("--num-speculative-tokens", type=int, default=0, help="draft tokens per step")
    ap.add_argument("--spec-method", choices=["mtp", "dflash"], default="mtp", help="drafter")
    ap.add_argument("--dflash-layers", type=int, default=1, help="DFlash drafter depth")
    ap.add_argument("--depth-policy", default="", help="dspark-depth-policy/1 file: per-request verify depth")
    ap.add_argument("--adaptive-k", default="", choices=["", "by_load", "accept"], help="adaptive draft count")
    ap.add_argument("--enforce-eager", action="store_true", help="no CUDA graphs")
    ap.add_argument("--nccl-collectives", action="store_true", help="TP collectives on NCCL (baseline path)")
    ap.add_argument("--no-warmup", action="store_true")
    ap.add_argument("--tool-call-parser", "--reasoning-parser", dest="parser", default=None,
                    choices=sorted(parsers.PARSERS),
                    help="reasoning / tool-call markup of the served model (glm45, glm47, ling3, deepseek_v41)")
    return ap.parse_args(argv)


def engine_config(args: argparse.Namespace) -> EngineConfig:
    """The engine configuration the server's command line describes."""
    from ..registry import resolve

    mcfg, _ckpt = resolve(args.model)
    return EngineConfig(model=mcfg,
                       parallel=ParallelConfig(tensor_parallel_size=args.tp, pipeline_parallel_size=args.pp,
                                               expert_parallel=args.enable_expert_parallel,
                                               fused_comm=not args.nccl_collectives),
                       scheduler=SchedulerConfig(max_num_seqs=args.max_num_seqs,
                                                 max_num_batched_tokens=args.max_num_batched_tokens,
                                                 max_model_len=args.max_model_len,
                                                 prefill_chunk_with_decodes=args.prefill_chunk_with_decodes,
                                                 max_num_partial_prefills=args.max_num_partial_prefills,
                                                 num_speculative_tokens=args.num_speculative_tokens,
                                                 spec_method=args.spec_method, dflash_layers=args.dflash_layers,
                                                 depth_policy=args.depth_policy, adaptive_k=args.adaptive_k),
                       cache=CacheConfig(), device=args.device, enforce_eager=args.enforce_eager)


def main(argv=None):
    args = parse_args(argv)
    from ..parallel import state as pstate

    st = pstate.init(tp_size=args.tp, pp_size=args.pp, device=args.device)
    cfg = engine_config(args)
    mcfg = cfg.model
    engine = LLMEngine(cfg)
    if st.tp_size > 1 and not args.nccl_collectives:
        from ..parallel import symm

        symm.enable_for_engine(engine)
    if not args.no_warmup:
        engine.warmup()
    tok = get_tokenizer(args.tokenizer, mcfg.vocab_size)
    engine.eos_token_id = getattr(tok, "eos_token_id", None)
    spmd = SPMDEngine(engine)
    if st.rank != 0:
        spmd.follow()
        return
    import uvicorn

    if args.parser in ("glm45", "glm47", "ling3"):
        from .. import envs

        envs.log_gate("tool_choice=none decode mask", bool(envs.get("VLLM_B200_TOOL_CHOICE_NONE_MASK")),
                      "VLLM_B200_TOOL_CHOICE_NONE_MASK")
    app = build_app(AsyncEngine(spmd), tok, args.model, parser=args.parser)
    uvicorn.run(app, host=args.host, port=args.port, log_level="info")


if __name__ == "__main__":
    main()
