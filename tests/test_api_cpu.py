"""HTTP API over the engine on CPU (tiny model): completions, chat with
reasoning + tool-call parsing, streaming, Anthropic messages, metrics; and
the parsers' recovery rules."""

import json

import pytest

from vllm_cmp170hx_b200.api import parsers


def test_parsers_reasoning_and_tools():
    r, c = parsers.split_reasoning("<think>plan</think>answer")
    assert (r, c) == ("plan", "answer")
    calls, content = parsers.parse_tool_calls('hi <tool_call>{"name": "f", "arguments": {"a": 1}}</tool_call>')
    assert content == "hi" and calls[0].name == "f" and calls[0].arguments == {"a": 1}
    # recovery: single quotes and trailing comma
    calls, _ = parsers.parse_tool_calls("<tool_call>{'name': 'g', 'arguments': {'x': 2,},}</tool_call>")
    assert calls and calls[0].name == "g" and calls[0].arguments == {"x": 2}
    # GLM argument tags
    calls, _ = parsers.parse_tool_calls("<tool_call>get<arg_key>city</arg_key><arg_value>\"Oslo\"</arg_value></tool_call>")
    assert calls[0].name == "get" and calls[0].arguments == {"city": "Oslo"}
    # unrecoverable call stays text
    calls, content = parsers.parse_tool_calls("<tool_call>{{{</tool_call>")
    assert not calls and "<tool_call>" in content


def test_streaming_parser_holds_back_partial_tags():
    sp = parsers.StreamingParser()
    out = [sp.feed(x) for x in ["<th", "ink>ab", "c</th", "ink>hello <tool", '_call>{"name":"f","arguments":{}}',
                                "</tool_call> bye"]]
    r = "".join(o[0] for o in out)
    c = "".join(o[1] for o in out) + sp.finish()[1]
    assert r == "abc" and c == "hello  bye" and sp.calls[0].name == "f"


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient

    from vllm_cmp170hx_b200.api.server import AsyncEngine, build_app
    from vllm_cmp170hx_b200.api.tokenizer import ByteTokenizer
    from vllm_cmp170hx_b200.config import CacheConfig, EngineConfig, SchedulerConfig, tiny
    from vllm_cmp170hx_b200.engine.llm_engine import LLMEngine
    from vllm_cmp170hx_b200.engine.spmd import SPMDEngine
    from vllm_cmp170hx_b200.parallel import state as pstate

    pstate.set_state(pstate.ParallelState())
    cfg = EngineConfig(model=tiny(layers=2, experts=4, expert_format="bf16"),
                       scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512),
                       cache=CacheConfig(num_blocks=32), device="cpu", enforce_eager=True)
    eng = LLMEngine(cfg)
    ae = AsyncEngine(SPMDEngine(eng))
    with TestClient(build_app(ae, ByteTokenizer(512), "tiny")) as c:
        yield c
    ae.shutdown()


def test_http_endpoints(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 3}).json()
    assert r["usage"]["completion_tokens"] == 3 and len(r["choices"][0]["token_ids"]) == 3
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 2}).json()
    assert r["usage"]["prompt_tokens"] == 3
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                   "max_tokens": 4}).json()
    assert r["choices"][0]["message"]["role"] == "assistant"
    with client.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                             "max_tokens": 3, "stream": True}) as s:
        lines = [l for l in s.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]" and json.loads(lines[-2][6:])["choices"][0]["finish_reason"] == "length"
    r = client.post("/v1/messages", json={"system": "be brief", "messages": [{"role": "user", "content": "hi"}],
                                          "max_tokens": 2}).json()
    assert r["type"] == "message" and r["usage"]["output_tokens"] == 2
    text = client.get("/metrics").text
    assert "b200_requests_total" in text and "b200_engine_steps_total" in text


def test_server_command_line_reaches_engine_config():
    from vllm_cmp170hx_b200.api.server import engine_config, parse_args

    args = parse_args(["--model", "tiny", "--device", "cpu", "--num-speculative-tokens", "3", "--spec-method", "dflash",
                       "--dflash-layers", "2", "--depth-policy", "/tmp/p.json", "--adaptive-k", "accept",
                       "--max-num-seqs", "8"])
    cfg = engine_config(args)
    sc = cfg.scheduler
    assert (sc.num_speculative_tokens, sc.spec_method, sc.dflash_layers, sc.depth_policy, sc.adaptive_k,
            sc.max_num_seqs) == (3, "dflash", 2, "/tmp/p.json", "accept", 8)


class _ScriptedEngine:
    """Stands in for the engine: records each request's sampling params and replies with a fixed
    text (byte tokens of the ByteTokenizer)."""

    def __init__(self, tok, text):
        self.tok, self.text, self.params = tok, text, []

    async def generate(self, ids, params):
        from types import SimpleNamespace

        self.params.append(params)
        out_ids = self.tok.encode(self.text)
        half = len(out_ids) // 2
        yield SimpleNamespace(new_token_ids=out_ids[:half], output_token_ids=out_ids[:half], finished=False,
                              finish_reason=None)
        yield SimpleNamespace(new_token_ids=out_ids[half:], output_token_ids=out_ids, finished=True,
                              finish_reason="stop")


@pytest.mark.parametrize("stream", [False, True])
def test_glm_parser_and_tool_choice_none_mask(monkeypatch, stream):
    from fastapi.testclient import TestClient

    from vllm_cmp170hx_b200 import envs
    from vllm_cmp170hx_b200.api.server import build_app
    from vllm_cmp170hx_b200.api.tokenizer import ByteTokenizer

    tok = ByteTokenizer(512)
    tok.special_ids = dict(tok.special_ids, **{"<tool_call>": 2})
    text = ("<think>look it up</think>On it.<tool_call>get_weather<arg_key>city</arg_key>"
            "<arg_value>Oslo</arg_value></tool_call>")
    eng = _ScriptedEngine(tok, text)
    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {
        "type": "object", "properties": {"city": {"type": "string"}}}}}]
    monkeypatch.setenv("VLLM_B200_TOOL_CHOICE_NONE_MASK", "1")
    envs._cache.clear()
    try:
        with TestClient(build_app(eng, tok, "glm", parser="glm47")) as c:
            body = {"messages": [{"role": "user", "content": "weather?"}], "tools": tools, "stream": stream}
            if stream:
                with c.stream("POST", "/v1/chat/completions", json=body) as s:
                    chunks = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: {")]
                deltas = [ch["choices"][0]["delta"] for ch in chunks]
                content = "".join(d.get("content", "") for d in deltas)
                reasoning = "".join(d.get("reasoning_content", "") for d in deltas)
                calls = [tc for d in deltas for tc in d.get("tool_calls", [])]
                fin = chunks[-1]["choices"][0]["finish_reason"]
            else:
                m = c.post("/v1/chat/completions", json=body).json()["choices"][0]
                content, reasoning = m["message"]["content"], m["message"]["reasoning_content"]
                calls, fin = m["message"]["tool_calls"], m["finish_reason"]
            assert (content, reasoning, fin) == ("On it.", "look it up", "tool_calls")
            assert [(t["function"]["name"], json.loads(t["function"]["arguments"])) for t in calls] == \
                [("get_weather", {"city": "Oslo"})]
            assert eng.params[-1].bad_token_ids == []
            # tool_choice="none": the opener is banned and the markup is not parsed as a call
            r = c.post("/v1/chat/completions", json=dict(body, tool_choice="none", stream=False)).json()
            assert eng.params[-1].bad_token_ids == [2]
            assert "tool_calls" not in r["choices"][0]["message"]
    finally:
        envs._cache.clear()
