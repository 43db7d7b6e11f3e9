"""Reasoning and tool-call parsers for chat completions.

Families, under the names the reference registers (vllm_sm80/parsers/__init__.py:20-41):

  * ``glm45`` / ``glm47``: GLM-4.7 markup, ``<tool_call>NAME<arg_key>K</arg_key><arg_value>V</arg_value>...
    </tool_call>`` (zero arguments allowed, the name on the opener's line), reasoning in
    ``<think>...</think>``.  Under ``tool_choice="none"`` with ``VLLM_B200_TOOL_CHOICE_NONE_MASK`` on, the
    tool-call opener token is banned at decode time (vllm_sm80/parsers/glm47.py:27-42), so the model
    cannot open a call the request does not allow.
  * ``ling3``: the GLM-4.7 markup and mask (vllm_sm80/parsers/ling3.py:14).
  * ``deepseek_v41``: DSML, ``<｜DSML｜tool_calls>`` around ``<｜DSML｜invoke name="N">`` with
    ``<｜DSML｜parameter name="P" string="true|false">V</｜DSML｜parameter>`` children, plus recovery of
    damaged calls (vllm_sm80/deepseek_v41_recovery.py:1-28):
      - near-miss wrapper spellings (``<｜DSML｜calls>``, ``<｜DSML｜_calls>``) parse as the wrapper;
      - a call in the plain XML idiom, ``<invoke name="TOOL">`` with plain or DSML parameter tags and a
        plain or DSML invoke closer, is a call when TOOL is a declared tool;
      - the invoke fused into its first parameter, ``<parameter name="TOOL">lead</parameter>...``:
        the lead value belongs to the tool's primary parameter;
      - a headless call, parameter tags only, up to an invoke closer: the tool is the single declared
        tool whose parameters cover every parameter written and that has all its required ones.
    A damaged candidate is held (never streamed) until its invoke closer arrives.  Outside parameter
    values it may hold only whitespace and call markup; the first other character, a name that is no
    declared tool, an ambiguous headless block or the end of the output restores it as text, and
    scanning resumes where it failed.  No candidate opens inside the thinking block, inside a Markdown
    code fence of the content, or under ``tool_choice="none"`` (then nothing is a call).
  * ``generic``: ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>`` JSON calls (or the GLM
    body), malformed JSON repaired in the common ways (single quotes, trailing commas, a missing
    closing brace, code fences) when the repair parses (vllm_sm80/parser_recovery.py:1-30 is the
    reference's provisional-call engine).

Every family is one left-to-right scanner over the generated text with a small state (inside the
thinking block, inside a call block, inside a code fence).  The streaming parser re-runs the scanner
from the last decided position on each delta, so text is emitted as soon as nothing later can change
its meaning; a possible tag prefix at the end is held back, and a held call leaks nothing.
"""

from __future__ import annotations

import json
import re
import uuid
from dataclasses import dataclass, field
from typing import Any, Iterable

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


@dataclass
class Parsed:
    reasoning: str | None
    content: str
    calls: list[ToolCall]


# ------------------------------------------------------------------------------------ declared tools
@dataclass(frozen=True)
class ToolSpec:
    name: str
    props: dict
    required: tuple


def tool_specs(tools: Iterable[Any] | None) -> list[ToolSpec]:
    """(name, properties, required) of every declared function (OpenAI ``{"type": "function",
    "function": {...}}`` entries or bare function dicts)."""
    out = []
    for t in tools or []:
        if not isinstance(t, dict):
            continue
        fn = t.get("function") if isinstance(t.get("function"), dict) else t
        name = fn.get("name")
        if not isinstance(name, str) or not name:
            continue
        params = fn.get("parameters") if isinstance(fn.get("parameters"), dict) else {}
        props = params.get("properties") if isinstance(params.get("properties"), dict) else {}
        out.append(ToolSpec(name, props, tuple(params.get("required") or ())))
    return out


def _prop_type(props: dict, name: str):
    p = props.get(name)
    if not isinstance(p, dict):
        return None
    t = p.get("type")
    if isinstance(t, list):  # ["string", "null"]
        t = next((x for x in t if x != "null"), None)
    return t


def _convert_value(raw: str, typ, string_attr: str | None = None):
    """A parameter's text as a JSON value: string-typed (by attribute or schema) stays text; anything
    else parses as JSON when it can, and stays text when it cannot."""
    if string_attr == "true":
        return raw
    if string_attr is None and typ == "string":
        return raw
    s = raw.strip()
    try:
        return json.loads(s)
    except (json.JSONDecodeError, ValueError):
        pass
    if typ in ("integer", "number"):
        try:
            return int(s) if typ == "integer" else float(s)
        except ValueError:
            return raw
    if typ == "boolean" and s.lower() in ("true", "false"):
        return s.lower() == "true"
    return raw


# ------------------------------------------------------------------------------------ scanner core
class _Need(Exception):
    """The scanner needs more text to decide what follows the current position."""


def _partial_tag(text: str, pos: int, tags: Iterable[str]) -> bool:
    """True if text[pos:] is a proper prefix of one of the tags (more text may complete it)."""
    rest = text[pos:]
    return any(len(rest) < len(t) and t.startswith(rest) for t in tags)


class _Scanner:
    """Base of the family scanners.  ``scan(text, final)`` returns the events of the decided part of
    ``text`` beyond the scanner's position and advances it; with ``final`` everything is decided."""

    tool_tags: tuple[str, ...] = ()

    def __init__(self, tools=None, tools_enabled: bool = True, reasoning: bool = True,
                 think_open_in_prompt: bool = False):
        self.specs = tool_specs(tools)
        self.tools_enabled = tools_enabled
        self.reasoning = reasoning
        self.pos = 0
        self.in_think = bool(think_open_in_prompt and reasoning)
        self.at_start = True  # a ``<think>`` opener counts only before any content
        self._fpos = 0  # fence state: the start of the first line not yet counted, and the state there
        self._fstate = False

    # events: ("reasoning", str) | ("content", str) | ("call", ToolCall)
    def scan(self, text: str, final: bool) -> list[tuple]:
        ev: list[tuple] = []
        while self.pos < len(text):
            try:
                if not self._step(text, final, ev):
                    break
            except _Need:
                if final:
                    self._flush_undecided(text, ev)
                break
        return _merge(ev)

    def _emit_text(self, ev, s: str):
        if not s:
            return
        if self.in_think:
            ev.append(("reasoning", s))
            return
        if s.strip():
            self.at_start = False
        ev.append(("content", s))

    def _fence_at(self, text: str, i: int) -> bool:
        """Whether position i of the content lies inside a Markdown code fence (from a line opening
        with ``` or ~~~ to the next such line).  Complete lines before i are counted once."""
        while True:
            nl = text.find("\n", self._fpos)
            if nl < 0 or nl >= i:
                break
            if _fence_line(text, self._fpos, nl):
                self._fstate = not self._fstate
            self._fpos = nl + 1
        return self._fstate != _fence_line(text, self._fpos, i)

    def _flush_undecided(self, text: str, ev):
        """The end of the output: text still undecided stays text."""
        self._emit_text(ev, text[self.pos:])
        self.pos = len(text)

    def _step(self, text: str, final: bool, ev) -> bool:
        """Consume one decided piece at self.pos; False when nothing more can be decided."""
        pos = self.pos
        if self.in_think:
            i = text.find(THINK_CLOSE, pos)
            if i < 0:
                hold = _holdback(text, pos, (THINK_CLOSE,)) if not final else len(text)
                self._emit_text(ev, text[pos:hold])
                self.pos = hold
                return final and hold < len(text)
            self._emit_text(ev, text[pos:i])
            self.in_think = False
            self.pos = i + len(THINK_CLOSE)
            self._fpos, self._fstate = self.pos, False  # fences count in the content only
            return True
        if self.reasoning and self.at_start:
            j = pos
            while j < len(text) and text[j].isspace():
                j += 1
            if j == len(text) and not final:
                return False
            if text.startswith(THINK_OPEN, j):
                self.in_think = True
                self.at_start = False
                self.pos = j + len(THINK_OPEN)
                return True
            if _partial_tag(text, j, (THINK_OPEN,)) and not final:
                return False
            if text.startswith(THINK_CLOSE, j):  # the template opened the block in the prompt
                self.pos = j + len(THINK_CLOSE)
                return True
        # content: find the next tag this family cares about
        tags = self._content_tags()
        i, tag = _find_first(text, pos, tags)
        if i < 0:
            hold = len(text) if final else _holdback(text, pos, tags)
            self._emit_text(ev, text[pos:hold])
            self.pos = hold
            return False
        self._emit_text(ev, text[pos:i])
        self.pos = i
        consumed = self._on_tag(text, i, tag, final, ev)
        if not consumed:  # the tag was text after all
            self._emit_text(ev, text[i])
            self.pos = i + 1
        return True

    def _content_tags(self) -> tuple[str, ...]:
        t = (THINK_CLOSE,) if self.reasoning else ()
        return t + (self.tool_tags if self.tools_enabled else ())

    def _on_tag(self, text, i, tag, final, ev) -> bool:
        if tag == THINK_CLOSE:  # a stray closer after content: drop it, keep the text around it
            self.pos = i + len(THINK_CLOSE)
            return True
        return False


def _fence_line(text: str, start: int, end: int) -> bool:
    j = start
    while j < end and text[j] in " \t":
        j += 1
    return j + 3 <= end and text[j:j + 3] in ("```", "~~~")


def _merge(ev):
    out = []
    for e in ev:
        if out and e[0] != "call" and out[-1][0] == e[0]:
            out[-1] = (e[0], out[-1][1] + e[1])
        else:
            out.append(e)
    return out


def _find_first(text: str, pos: int, tags: Iterable[str]) -> tuple[int, str | None]:
    best, best_tag = -1, None
    for t in tags:
        i = text.find(t, pos)
        if i >= 0 and (best < 0 or i < best):
            best, best_tag = i, t
    return best, best_tag


def _holdback(text: str, pos: int, tags: Iterable[str]) -> int:
    """The end of the part of text[pos:] that no tag can still start in."""
    end = len(text)
    for t in tags:
        for k in range(min(len(t) - 1, end - pos), 0, -1):
            if text.endswith(t[:k]):
                end = min(end, len(text) - k)
                break
    return max(end, pos)


# ------------------------------------------------------------------------------------ generic JSON
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


_GLM_ARG = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)
_GLM_BODY = re.compile(r"\s*([^\s<]+?)\s*(<arg_key>.*)?\s*$", re.S)


def _parse_glm_body(body: str, specs: list[ToolSpec], require_declared: bool) -> ToolCall | None:
    m = _GLM_BODY.match(body)
    if not m:
        return None
    name, rest = m.group(1), m.group(2) or ""
    spec = next((s for s in specs if s.name == name), None)
    if require_declared and specs and spec is None:
        return None
    props = spec.props if spec else {}
    args = {}
    pos = 0
    for am in _GLM_ARG.finditer(rest):
        if rest[pos:am.start()].strip():
            return None  # text between arguments: not a call
        k = am.group(1).strip()
        args[k] = _convert_value(am.group(2), _prop_type(props, k)) if spec else _json_or_text(am.group(2))
        pos = am.end()
    if rest[pos:].strip():
        return None
    return ToolCall(name, args)


def _json_or_text(v: str):
    try:
        return json.loads(v)
    except json.JSONDecodeError:
        return v


def _parse_generic_body(body: str, specs: list[ToolSpec]) -> ToolCall | None:
    body = body.strip()
    if body.startswith("{"):
        obj = _repair_json(body)
        if isinstance(obj, dict) and isinstance(obj.get("name"), str):
            args = obj.get("arguments", obj.get("parameters", {}))
            if isinstance(args, str):
                args = _repair_json(args) or {"_raw": args}
            return ToolCall(obj["name"], args if isinstance(args, dict) else {"value": args})
        return None
    return _parse_glm_body(body, specs, require_declared=False)


class _TagCallScanner(_Scanner):
    """``<tool_call>BODY</tool_call>`` calls (the generic and GLM families)."""

    tool_tags = (CALL_OPEN,)
    require_declared = False

    def _parse_body(self, body: str) -> ToolCall | None:
        raise NotImplementedError

    def _on_tag(self, text, i, tag, final, ev) -> bool:
        if tag != CALL_OPEN:
            return super()._on_tag(text, i, tag, final, ev)
        j = text.find(CALL_CLOSE, i + len(CALL_OPEN))
        if j < 0:
            if not final:
                raise _Need
            call = self._parse_body(text[i + len(CALL_OPEN):])  # truncated final call
            if call is None:
                return False
            ev.append(("call", call))
            self.pos = len(text)
            return True
        call = self._parse_body(text[i + len(CALL_OPEN):j])
        if call is None:  # unrecoverable: the whole block stays text
            self._emit_text(ev, text[i:j + len(CALL_CLOSE)])
        else:
            ev.append(("call", call))
        self.at_start = False
        self.pos = j + len(CALL_CLOSE)
        return True

    def _flush_undecided(self, text, ev):
        # the end of the output inside an unclosed call: try it as a truncated call
        if self.tools_enabled and text.startswith(CALL_OPEN, self.pos):
            call = self._parse_body(text[self.pos + len(CALL_OPEN):])
            if call is not None:
                ev.append(("call", call))
                self.pos = len(text)
                return
        super()._flush_undecided(text, ev)


class GenericScanner(_TagCallScanner):
    def _parse_body(self, body):
        return _parse_generic_body(body, self.specs)


class Glm47Scanner(_TagCallScanner):
    require_declared = True

    def _parse_body(self, body):
        return _parse_glm_body(body, self.specs, require_declared=True)


# ------------------------------------------------------------------------------------ DSML
D = "｜DSML｜"
DSML_WRAPPERS = (f"<{D}tool_calls>", f"<{D}function_calls>", f"<{D}calls>", f"<{D}_calls>")
DSML_WRAPPER_CLOSERS = tuple("</" + w[1:] for w in DSML_WRAPPERS)
DSML_INVOKE = f'<{D}invoke name="'
XML_INVOKE = '<invoke name="'
XML_PARAM = '<parameter name="'
# parameter tags of any spelling: DSML, plain or mixed (a space after the marker tolerated), the
# string attribute optional
_P_OPEN = re.compile(rf'<(?:{D} ?)?parameter\s+name="([^"<>]+)"(?:\s+string="(true|false)")?\s*>')
_P_CLOSE = re.compile(rf"</(?:{D} ?)?parameter>")
_INVOKE_OPEN = re.compile(rf'<(?:{D} ?)?invoke\s+name="([^"<>]*)"\s*>')
_INVOKE_CLOSE = re.compile(rf"</(?:{D} ?)?invoke>")
_BLOCK_CLOSE = re.compile(rf"</(?:{D} ?)?(?:tool_calls|function_calls|calls|_calls)>")
_NAME_LIMIT = 256  # a longer "name" is prose quoting an opener
_TAG_LIMIT = 320  # a tag still arriving is waited for up to this length


def _primary_param(spec: ToolSpec) -> str | None:
    """The parameter a fused invoke's leading value belongs to: the first required string (or
    untyped) parameter, else the first required one, else the first string one, else the first."""
    for n in spec.required:
        if n in spec.props and _prop_type(spec.props, n) in (None, "string"):
            return n
    for n in spec.required:
        if n in spec.props:
            return n
    for n in spec.props:
        if _prop_type(spec.props, n) == "string":
            return n
    if spec.props:
        return next(iter(spec.props))
    return spec.required[0] if spec.required else None


class _ParamBody:
    """Parse a run of parameter tags (any spelling) starting at ``pos`` up to an invoke closer.

    Returns (params [(name, string_attr, raw)], lead value or None, end of the closer) or raises
    _Need; returns None when the text stops looking like a call (``shape`` violations)."""

    @staticmethod
    def parse(text: str, pos: int, final: bool, lead: bool):
        params: list[tuple[str, str | None, str]] = []
        lead_val = None
        i = pos
        if lead:  # a fused invoke: the leading value runs to its own closer
            m_close = _P_CLOSE.search(text, i)
            m_open = _P_OPEN.search(text, i)
            m_end = _INVOKE_CLOSE.search(text, i)
            stops = [m for m in (m_close, m_open, m_end) if m is not None]
            if not stops:
                if final:
                    return None
                raise _Need
            first = min(stops, key=lambda m: m.start())
            lead_val = text[i:first.start()]
            i = first.end() if first is m_close else first.start()
        while True:
            while i < len(text) and text[i].isspace():
                i += 1
            if i >= len(text):
                if final:
                    return None
                raise _Need
            if text[i] != "<":
                return None
            m = _INVOKE_CLOSE.match(text, i)
            if m:
                return params, lead_val, m.end()
            m = _P_OPEN.match(text, i)
            if m:
                start = m.end()
                # a value ends at its own closer when one comes before the next opener (a value may
                # quote call markup), else at the next opener or invoke closer
                c = _P_CLOSE.search(text, start)
                o = _P_OPEN.search(text, start)
                if c is not None and (o is None or c.start() < o.start()):
                    params.append((m.group(1), m.group(2), text[start:c.start()]))
                    i = c.end()
                    continue
                e = _INVOKE_CLOSE.search(text, start)
                ends = [x.start() for x in (o, e) if x is not None]
                if not ends:
                    if final:
                        return None
                    raise _Need
                params.append((m.group(1), m.group(2), text[start:min(ends)]))
                i = min(ends)
                continue
            # a tag that may still be arriving
            if text.find(">", i) < 0 and len(text) - i <= _TAG_LIMIT and not final:
                raise _Need
            return None


class DeepSeekV41Scanner(_Scanner):
    """DSML calls with damaged-call recovery."""

    tool_tags = DSML_WRAPPERS + (XML_INVOKE, XML_PARAM, DSML_INVOKE)

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.in_block = False  # between a wrapper and its closer

    def _content_tags(self):
        if self.in_block:
            return ()
        return super()._content_tags()

    def _step(self, text, final, ev) -> bool:
        if not self.in_block:
            return super()._step(text, final, ev)
        # inside a proper (or near-miss) wrapper: invokes, whitespace, the closer
        i = self.pos
        while i < len(text) and text[i].isspace():
            i += 1
        if i >= len(text):
            if final:
                self.in_block = False
                self.pos = len(text)
                return False
            raise _Need
        m = _BLOCK_CLOSE.match(text, i)
        if m:
            self.in_block = False
            self.pos = m.end()
            return True
        m = _INVOKE_OPEN.match(text, i)
        if m:
            call, end = self._finish_invoke(text, m.group(1), m.end(), final, declared_only=False)
            if call is None:  # a broken invoke inside the block: the block ends, its text is content
                self.in_block = False
                self._emit_text(ev, text[self.pos:i + 1])
                self.pos = i + 1
                return True
            ev.append(("call", call))
            self.pos = end
            return True
        if not final and (_partial_tag(text, i, ("</",) + tuple(DSML_WRAPPER_CLOSERS) + (DSML_INVOKE, XML_INVOKE))
                          or (text.find(">", i) < 0 and len(text) - i <= _TAG_LIMIT)):
            raise _Need
        # other text inside the block: leave the block, the text is content
        self.in_block = False
        self.pos = i
        return True

    def _flush_undecided(self, text, ev):
        self.in_block = False
        super()._flush_undecided(text, ev)

    def _spec(self, name: str) -> ToolSpec | None:
        return next((s for s in self.specs if s.name == name), None)

    def _finish_invoke(self, text, name, body_start, final, declared_only: bool, lead: bool = False):
        res = _ParamBody.parse(text, body_start, final, lead)
        if res is None:
            return None, body_start
        params, lead_val, end = res
        spec = self._spec(name)
        if spec is None and declared_only:
            return None, body_start
        return self._make_call(name, spec, params, lead_val), end

    def _make_call(self, name, spec, params, lead_val) -> ToolCall:
        props = spec.props if spec else {}
        args: dict[str, Any] = {}
        if lead_val is not None and lead_val.strip() and spec is not None:
            p = _primary_param(spec)
            if p is not None:
                args[p] = _convert_value(lead_val.strip(), _prop_type(props, p))
        for pname, sattr, raw in params:
            args[pname] = _convert_value(raw, _prop_type(props, pname), sattr)
        return ToolCall(name, _unwrap_args(args, spec))

    def _on_tag(self, text, i, tag, final, ev) -> bool:
        if tag in DSML_WRAPPERS:
            self.in_block = True
            self.at_start = False
            self.pos = i + len(tag)
            return True
        if tag == DSML_INVOKE:  # a DSML invoke without its wrapper: parse it the proper way
            m = _INVOKE_OPEN.match(text, i)
            if m is None:
                if not final and text.find(">", i) < 0 and len(text) - i <= _TAG_LIMIT:
                    raise _Need
                return False
            call, end = self._finish_invoke(text, m.group(1), m.end(), final, declared_only=False)
            if call is None:
                return False
            ev.append(("call", call))
            self.at_start = False
            self.pos = end
            return True
        if tag in (XML_INVOKE, XML_PARAM):
            if not self.specs or self._fence_at(text, i):
                return False
            return self._recover(text, i, tag, final, ev)
        return super()._on_tag(text, i, tag, final, ev)

    def _recover(self, text, i, tag, final, ev) -> bool:
        """A damaged call opened by a plain invoke or parameter tag: held until decided."""
        name_start = i + len(tag)
        q = text.find('"', name_start)
        if q < 0:
            if len(text) - name_start > _NAME_LIMIT or final:
                return False
            raise _Need
        name = text[name_start:q]
        if len(name) > _NAME_LIMIT or "\n" in name or "<" in name:
            return False
        if tag == XML_INVOKE:
            m = _INVOKE_OPEN.match(text, i)
            if m is None:
                if not final and text.find(">", q) < 0 and len(text) - q <= _TAG_LIMIT:
                    raise _Need
                return False
            if self._spec(name) is None:  # the name ends: it must be a declared tool
                self._emit_text(ev, text[i:m.end()])
                self.pos = m.end()
                return True
            call, end = self._finish_invoke(text, name, m.end(), final, declared_only=True)
        else:
            m = _P_OPEN.match(text, i)
            if m is None:
                if not final and text.find(">", q) < 0 and len(text) - q <= _TAG_LIMIT:
                    raise _Need
                return False
            if self._spec(name) is not None:  # the invoke fused into its first parameter
                call, end = self._finish_invoke(text, name, m.end(), final, declared_only=True, lead=True)
            else:  # headless: the opener is the first parameter
                res = _ParamBody.parse(text, i, final, lead=False)
                call, end = None, i
                if res is not None:
                    params, _, end = res
                    spec = self._headless_tool({p[0] for p in params})
                    if spec is not None:
                        call = self._make_call(spec.name, spec, params, None)
        if call is None:
            return False
        ev.append(("call", call))
        self.at_start = False
        self.pos = end
        return True

    def _headless_tool(self, names: set) -> ToolSpec | None:
        if not names:
            return None
        covering = [s for s in self.specs if s.props and names <= s.props.keys()]
        if len(covering) != 1 or not set(covering[0].required) <= names:
            return None
        return covering[0]


def _unwrap_args(args: dict, spec: ToolSpec | None) -> dict:
    """Arguments the model wrapped in one ``arguments``/``parameters`` object that the tool does not
    declare are unwrapped."""
    if len(args) == 1 and spec is not None:
        (k, v), = args.items()
        if k in ("arguments", "parameters", "input") and k not in spec.props and isinstance(v, dict):
            return v
    return args


# ------------------------------------------------------------------------------------ registry
@dataclass(frozen=True)
class Family:
    name: str
    scanner: type
    # the tool-call opener banned at decode time under tool_choice="none" (None: no mask)
    mask_token: str | None = None


PARSERS: dict[str, Family] = {
    "generic": Family("generic", GenericScanner),
    "glm45": Family("glm45", Glm47Scanner, CALL_OPEN),
    "glm47": Family("glm47", Glm47Scanner, CALL_OPEN),
    "ling3": Family("ling3", Glm47Scanner, CALL_OPEN),
    "deepseek_v41": Family("deepseek_v41", DeepSeekV41Scanner),
}


def get_family(name: str | None) -> Family:
    if not name:
        return PARSERS["generic"]
    if name not in PARSERS:
        raise ValueError(f"unknown parser {name!r}; known: {sorted(PARSERS)}")
    return PARSERS[name]


def tools_enabled(body: dict) -> bool:
    return bool(body.get("tools")) and body.get("tool_choice", "auto") != "none"


def tool_choice_none_bans(family: Family, body: dict, tokenizer) -> list[int]:
    """Token ids to ban at decode time for this request: the family's tool-call opener, when the
    request says ``tool_choice="none"``, the mask flag is on and the opener is one token."""
    from .. import envs

    if family.mask_token is None or body.get("tool_choice") != "none" or not envs.get("VLLM_B200_TOOL_CHOICE_NONE_MASK"):
        return []
    tid = token_id_of(tokenizer, family.mask_token)
    return [] if tid is None else [tid]


def token_id_of(tokenizer, text: str) -> int | None:
    special = getattr(tokenizer, "special_ids", None)
    if isinstance(special, dict) and text in special:
        return int(special[text])
    conv = getattr(getattr(tokenizer, "tok", None), "convert_tokens_to_ids", None)
    if conv is not None:
        tid = conv(text)
        unk = getattr(tokenizer.tok, "unk_token_id", None)
        if isinstance(tid, int) and tid != unk:
            return tid
    ids = tokenizer.encode(text)
    return int(ids[0]) if len(ids) == 1 else None


def parse(text: str, family: str | Family | None = None, tools=None, tool_choice: str = "auto",
          think_open_in_prompt: bool = False) -> Parsed:
    """Whole-output parse: (reasoning, content, calls)."""
    fam = family if isinstance(family, Family) else get_family(family)
    sc = fam.scanner(tools, tools_enabled=_calls_on(fam, tools, tool_choice), think_open_in_prompt=think_open_in_prompt)
    return _collect(sc.scan(text, final=True))


def _calls_on(fam: Family, tools, tool_choice: str) -> bool:
    """Calls are parsed when the request declares tools and allows them (the generic family also
    without declared tools)."""
    return tool_choice != "none" and (bool(tools) or fam.name == "generic")


def _collect(events) -> Parsed:
    r, c, calls = [], [], []
    for kind, v in events:
        (r if kind == "reasoning" else c if kind == "content" else calls).append(v)
    reasoning = "".join(r).strip() if r else None
    return Parsed(reasoning or None, "".join(c).strip(), calls)


class StreamParser:
    """Incremental parse: ``feed(delta)`` returns (reasoning delta, content delta, new calls);
    ``finish()`` the same for what is still held at the end of the output."""

    def __init__(self, family: str | Family | None = None, tools=None, tool_choice: str = "auto",
                 think_open_in_prompt: bool = False, tools_on: bool | None = None):
        fam = family if isinstance(family, Family) else get_family(family)
        on = _calls_on(fam, tools, tool_choice) if tools_on is None else tools_on
        self.sc = fam.scanner(tools, tools_enabled=on, think_open_in_prompt=think_open_in_prompt)
        self.text = ""
        self.calls: list[ToolCall] = []
        self._stripped_lead = False

    def _split(self, events):
        r, c, calls = "", "", []
        for kind, v in events:
            if kind == "reasoning":
                r += v
            elif kind == "content":
                c += v
            else:
                calls.append(v)
        if not self._stripped_lead and c:  # the content starts at its first non-space character
            c = c.lstrip()
            self._stripped_lead = bool(c)
        self.calls += calls
        return r, c, calls

    def feed(self, delta: str):
        self.text += delta
        return self._split(self.sc.scan(self.text, final=False))

    def finish(self):
        return self._split(self.sc.scan(self.text, final=True))


# ------------------------------------------------------------------------------------ compatibility
def split_reasoning(text: str) -> tuple[str | None, str]:
    """(reasoning, rest) of a whole output (``<think>`` opened in the output or by the template)."""
    if THINK_OPEN in text:
        pre, rest = text.split(THINK_OPEN, 1)
        if THINK_CLOSE in rest:
            r, post = rest.split(THINK_CLOSE, 1)
            return r.strip(), (pre + post).strip()
        return rest.strip(), pre.strip()
    if THINK_CLOSE in text:
        r, post = text.split(THINK_CLOSE, 1)
        return r.strip(), post.strip()
    return None, text


def parse_tool_calls(text: str) -> tuple[list[ToolCall], str]:
    """Generic-family calls of a whole output: (calls, remaining content)."""
    sc = GenericScanner(None, tools_enabled=True, reasoning=False)
    p = _collect(sc.scan(text, final=True))
    return p.calls, p.content


class StreamingParser:
    """Generic-family stream: ``feed`` returns (reasoning delta, content delta); calls collect in
    ``calls``."""

    def __init__(self, reasoning: bool = True, tools: bool = True):
        self.sc = GenericScanner(None, tools_enabled=tools, reasoning=reasoning)
        self.text = ""
        self.calls: list[ToolCall] = []

    def _split(self, events):
        r = "".join(v for k, v in events if k == "reasoning")
        c = "".join(v for k, v in events if k == "content")
        self.calls += [v for k, v in events if k == "call"]
        return r, c

    def feed(self, delta: str) -> tuple[str, str]:
        self.text += delta
        return self._split(self.sc.scan(self.text, final=False))

    def finish(self) -> tuple[str, str]:
        return self._split(self.sc.scan(self.text, final=True))
