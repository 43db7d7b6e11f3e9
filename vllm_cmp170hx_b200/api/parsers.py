"""Reasoning and tool-call parsers for chat completions, with recovery of
near-miss tool calls.

Formats (the families the reference registers, vllm_sm80/parsers/__init__.py:
GLM-4.7 / Ling3 XML-ish tags and DeepSeek-V4.1 DSML):
  * reasoning:  ``<think> ... </think>`` before the answer;
  * tool calls: ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``,
    or GLM's ``<tool_call>name<arg_key>k</arg_key><arg_value>v</arg_value>...</tool_call>``.
Recovery (vllm_sm80/parser_recovery.py): a call whose JSON is malformed in a
common way (single quotes, trailing commas, a missing closing brace, code
fences) is repaired when the repair parses; otherwise its text stays in the
content.  The streaming parser holds text back while it may still be the
start of a tag, so a provisional tool call never leaks into content.
"""

from __future__ import annotations

import json
import re
import uuid
from dataclasses import dataclass, field

THINK_OPEN, THINK_CLOSE = "<think>", "</think>"
CALL_OPEN, CALL_CLOSE = "<tool_call>", "</tool_call>"


@dataclass
class ToolCall:
    name: str
    arguments: dict
    id: str = field(default_factory=lambda: "call_" + uuid.uuid4().hex[:16])

    def to_openai(self) -> dict:
        return {"id": self.id, "type": "function",
                "function": {"name": self.name, "arguments": json.dumps(self.arguments, ensure_ascii=False)}}


def split_reasoning(text: str) -> tuple[str | None, str]:
    if THINK_OPEN in text:
        pre, rest = text.split(THINK_OPEN, 1)
        if THINK_CLOSE in rest:
            r, post = rest.split(THINK_CLOSE, 1)
            return r.strip(), (pre + post).strip()
        return rest.strip(), pre.strip()
    if THINK_CLOSE in text:  # template opened the block in the prompt
        r, post = text.split(THINK_CLOSE, 1)
        return r.strip(), post.strip()
    return None, text


def _repair_json(s: str):
    s = s.strip()
    s = re.sub(r"^```(?:json)?|```$", "", s).strip()
    for cand in (s, s.replace("'", '"'), re.sub(r",\s*([}\]])", r"\1", s), s + "}", s + "}}"):
        try:
            return json.loads(cand)
        except json.JSONDecodeError:
            continue
    fixed = re.sub(r",\s*([}\]])", r"\1", s.replace("'", '"'))
    for cand in (fixed, fixed + "}", fixed + "}}"):
        try:
            return json.loads(cand)
        except json.JSONDecodeError:
            continue
    return None


def _parse_call(body: str) -> ToolCall | None:
    body = body.strip()
    if body.startswith("{"):
        obj = _repair_json(body)
        if isinstance(obj, dict) and isinstance(obj.get("name"), str):
            args = obj.get("arguments", obj.get("parameters", {}))
            if isinstance(args, str):
                args = _repair_json(args) or {"_raw": args}
            return ToolCall(obj["name"], args if isinstance(args, dict) else {"value": args})
        return None
    # GLM style: name<arg_key>k</arg_key><arg_value>v</arg_value>...
    m = re.match(r"([\w.\-]+)", body)
    if not m:
        return None
    args = {}
    for k, v in re.findall(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", body, re.S):
        try:
            args[k.strip()] = json.loads(v)
        except json.JSONDecodeError:
            args[k.strip()] = v
    return ToolCall(m.group(1), args)


def parse_tool_calls(text: str) -> tuple[list[ToolCall], str]:
    """Extract complete tool calls; returns (calls, remaining content)."""
    calls, content, pos = [], [], 0
    for m in re.finditer(re.escape(CALL_OPEN) + r"(.*?)" + re.escape(CALL_CLOSE), text, re.S):
        content.append(text[pos:m.start()])
        call = _parse_call(m.group(1))
        if call is None:
            content.append(m.group(0))  # unrecoverable: keep as text
        else:
            calls.append(call)
        pos = m.end()
    rest = text[pos:]
    if CALL_OPEN in rest:  # truncated final call: try to recover it
        head, body = rest.split(CALL_OPEN, 1)
        call = _parse_call(body)
        if call is not None:
            calls.append(call)
            rest = head
    content.append(rest)
    return calls, "".join(content).strip()


class StreamingParser:
    """Incremental split of generated text into reasoning / content deltas;
    tool-call blocks are buffered until closed (or the stream ends)."""

    def __init__(self, reasoning: bool = True, tools: bool = True):
        self.buf = ""
        self.in_think = False
        self.reasoning = reasoning
        self.tools = tools
        self.calls: list[ToolCall] = []

    def _holdback(self, s: str) -> int:
        tags = [THINK_OPEN, THINK_CLOSE, CALL_OPEN]
        best = 0
        for t in tags:
            for k in range(1, len(t)):
                if s.endswith(t[:k]):
                    best = max(best, k)
        return best

    def feed(self, delta: str) -> tuple[str, str]:
        """Returns (reasoning_delta, content_delta)."""
        self.buf += delta
        r_out, c_out = "", ""
        while True:
            if self.in_think:
                i = self.buf.find(THINK_CLOSE)
                if i < 0:
                    hb = self._holdback(self.buf)
                    r_out += self.buf[: len(self.buf) - hb]
                    self.buf = self.buf[len(self.buf) - hb:]
                    return r_out, c_out
                r_out += self.buf[:i]
                self.buf = self.buf[i + len(THINK_CLOSE):]
                self.in_think = False
                continue
            if self.reasoning and self.buf.startswith(THINK_OPEN):
                self.buf = self.buf[len(THINK_OPEN):]
                self.in_think = True
                continue
            if self.tools and CALL_OPEN in self.buf:
                i = self.buf.find(CALL_OPEN)
                c_out += self.buf[:i]
                j = self.buf.find(CALL_CLOSE, i)
                if j < 0:
                    self.buf = self.buf[i:]
                    return r_out, c_out
                call = _parse_call(self.buf[i + len(CALL_OPEN):j])
                if call is not None:
                    self.calls.append(call)
                else:
                    c_out += self.buf[i:j + len(CALL_CLOSE)]
                self.buf = self.buf[j + len(CALL_CLOSE):]
                continue
            hb = self._holdback(self.buf)
            c_out += self.buf[: len(self.buf) - hb]
            self.buf = self.buf[len(self.buf) - hb:]
            return r_out, c_out

    def finish(self) -> tuple[str, str]:
        rest, self.buf = self.buf, ""
        if self.tools and rest.startswith(CALL_OPEN):
            calls, content = parse_tool_calls(rest)
            self.calls += calls
            return "", content
        return (rest, "") if self.in_think else ("", rest)
