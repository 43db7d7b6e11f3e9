"""Model-specific chat parsers: GLM-4.7 / Ling3 markup with the tool_choice="none" decode mask, and
DeepSeek-V4.1 DSML with damaged-call recovery.  Every case is parsed whole and streamed one character
at a time; both must agree, and a stream never leaks call markup into its content deltas."""

import pytest

from vllm_cmp170hx_b200.api import parsers as P

D = "｜DSML｜"
WEATHER = {"type": "function", "function": {"name": "get_weather", "parameters": {
    "type": "object", "properties": {"city": {"type": "string"}, "days": {"type": "integer"}},
    "required": ["city"]}}}
SEARCH = {"type": "function", "function": {"name": "search", "parameters": {
    "type": "object", "properties": {"query": {"type": "string"}, "limit": {"type": "integer"}},
    "required": ["query"]}}}
TOOLS = [WEATHER, SEARCH]


def _stream(text, family, tools=TOOLS, tool_choice="auto", step=1, think_open_in_prompt=False):
    sp = P.StreamParser(family, tools, tool_choice, think_open_in_prompt=think_open_in_prompt)
    r, c, calls = "", "", []
    for i in range(0, len(text), step):
        dr, dc, dcalls = sp.feed(text[i:i + step])
        r, c, calls = r + dr, c + dc, calls + dcalls
    dr, dc, dcalls = sp.finish()
    return r + dr, c + dc, calls + dcalls


def _check(text, family, tools=TOOLS, tool_choice="auto", **kw):
    whole = P.parse(text, family, tools, tool_choice, **kw)
    for step in (1, 3, 7):
        r, c, calls = _stream(text, family, tools, tool_choice, step, **kw)
        assert [(x.name, x.arguments) for x in calls] == [(x.name, x.arguments) for x in whole.calls], step
        assert (r.strip() or None) == whole.reasoning, step
        assert c.strip() == whole.content, step
    return whole


# ---------------------------------------------------------------------------------------- GLM-4.7
def test_glm47_call_with_typed_arguments():
    text = ("<think>need weather</think>Let me check."
            "<tool_call>get_weather<arg_key>city</arg_key><arg_value>Oslo</arg_value>"
            "<arg_key>days</arg_key><arg_value>3</arg_value></tool_call>")
    p = _check(text, "glm47")
    assert p.reasoning == "need weather"
    assert p.content == "Let me check."
    assert [(c.name, c.arguments) for c in p.calls] == [("get_weather", {"city": "Oslo", "days": 3})]


def test_glm47_string_parameter_keeps_json_looking_text():
    text = "<tool_call>search\n<arg_key>query</arg_key>\n<arg_value>123</arg_value>\n</tool_call>"
    p = _check(text, "glm47")
    assert p.calls[0].arguments == {"query": "123"}  # declared a string: not turned into a number


def test_glm47_zero_argument_call_and_two_calls():
    tools = TOOLS + [{"type": "function", "function": {"name": "now", "parameters": {"type": "object"}}}]
    text = "<tool_call>now</tool_call><tool_call>search<arg_key>query</arg_key><arg_value>b200</arg_value></tool_call>"
    p = _check(text, "glm47", tools)
    assert [(c.name, c.arguments) for c in p.calls] == [("now", {}), ("search", {"query": "b200"})]


def test_glm47_undeclared_tool_stays_text():
    text = "x <tool_call>rm_rf<arg_key>path</arg_key><arg_value>/</arg_value></tool_call>"
    p = _check(text, "glm47")
    assert p.calls == [] and "<tool_call>rm_rf" in p.content


def test_glm47_tool_choice_none_keeps_markup_as_content():
    text = "<tool_call>get_weather<arg_key>city</arg_key><arg_value>Oslo</arg_value></tool_call>"
    p = _check(text, "glm47", tool_choice="none")
    assert p.calls == [] and p.content == text


def test_ling3_is_glm47_markup():
    text = "<tool_call>get_weather<arg_key>city</arg_key><arg_value>Rome</arg_value></tool_call>"
    assert _check(text, "ling3").calls[0].arguments == {"city": "Rome"}
    assert P.get_family("ling3").mask_token == P.CALL_OPEN
    assert P.get_family("glm45").mask_token == P.CALL_OPEN
    assert P.get_family("deepseek_v41").mask_token is None


def test_reasoning_opened_by_the_template():
    p = _check("plan here</think>answer", "glm47", think_open_in_prompt=True)
    assert p.reasoning == "plan here" and p.content == "answer"


class _Tok:
    special_ids = {"<tool_call>": 151352}

    def encode(self, s):
        return [ord(ch) for ch in s]


@pytest.mark.parametrize("flag,choice,family,expect", [
    ("1", "none", "glm47", [151352]), ("1", "none", "ling3", [151352]), ("0", "none", "glm47", []),
    ("1", "auto", "glm47", []), ("1", "none", "deepseek_v41", []), ("1", "none", "generic", []),
])
def test_tool_choice_none_mask(monkeypatch, flag, choice, family, expect):
    from vllm_cmp170hx_b200 import envs

    monkeypatch.setenv("VLLM_B200_TOOL_CHOICE_NONE_MASK", flag)
    envs._cache.clear()
    try:
        got = P.tool_choice_none_bans(P.get_family(family), {"tool_choice": choice, "tools": TOOLS}, _Tok())
    finally:
        envs._cache.clear()
    assert got == expect


def test_mask_flag_reference_alias(monkeypatch):
    from vllm_cmp170hx_b200 import envs

    monkeypatch.delenv("VLLM_B200_TOOL_CHOICE_NONE_MASK", raising=False)
    monkeypatch.setenv("VLLM_TOOL_CHOICE_NONE_MASK", "1")
    envs._cache.clear()
    try:
        assert envs.get("VLLM_B200_TOOL_CHOICE_NONE_MASK") is True
    finally:
        envs._cache.clear()


# ---------------------------------------------------------------------------------------- DSML
def _dsml_call(name, params, wrapper="tool_calls"):
    body = "".join(f'<{D}parameter name="{k}" string="{s}">{v}</{D}parameter>\n' for k, v, s in params)
    return f'<{D}{wrapper}>\n<{D}invoke name="{name}">\n{body}</{D}invoke>\n</{D}{wrapper}>'


def test_dsml_proper_calls():
    text = "Checking." + _dsml_call("get_weather", [("city", "杭州", "true"), ("days", "2", "false")])
    p = _check(text, "deepseek_v41")
    assert p.content == "Checking."
    assert [(c.name, c.arguments) for c in p.calls] == [("get_weather", {"city": "杭州", "days": 2})]


def test_dsml_two_invokes_in_one_block_and_function_calls_spelling():
    inv = lambda c: f'<{D}invoke name="get_weather"><{D}parameter name="city" string="true">{c}</{D}parameter></{D}invoke>'
    text = f"<{D}function_calls>\n{inv('A')}\n{inv('B')}\n</{D}function_calls> done"
    p = _check(text, "deepseek_v41")
    assert [c.arguments["city"] for c in p.calls] == ["A", "B"] and p.content == "done"


@pytest.mark.parametrize("wrapper", ["calls", "_calls"])
def test_dsml_near_miss_wrapper(wrapper):
    p = _check(_dsml_call("search", [("query", "nvlink", "true")], wrapper), "deepseek_v41")
    assert [(c.name, c.arguments) for c in p.calls] == [("search", {"query": "nvlink"})]
    assert p.content == ""


def test_xml_idiom_call_of_a_declared_tool():
    text = 'Sure. <invoke name="get_weather">\n<parameter name="city">Paris</parameter>\n<parameter name="days">4</parameter>\n</invoke>'
    p = _check(text, "deepseek_v41")
    assert p.content == "Sure."
    assert [(c.name, c.arguments) for c in p.calls] == [("get_weather", {"city": "Paris", "days": 4})]


def test_xml_idiom_mixed_closers():
    text = f'<invoke name="search"><{D}parameter name="query" string="true">x</{D}parameter></{D}invoke>'
    p = _check(text, "deepseek_v41")
    assert [(c.name, c.arguments) for c in p.calls] == [("search", {"query": "x"})]


def test_xml_idiom_undeclared_name_stays_text():
    text = 'see <invoke name="format_disk"><parameter name="dev">sda</parameter></invoke>'
    p = _check(text, "deepseek_v41")
    assert p.calls == [] and p.content == text


def test_fused_invoke_lead_value_goes_to_primary_parameter():
    text = '<parameter name="get_weather">Berlin</parameter><parameter name="days">2</parameter></invoke>'
    p = _check(text, "deepseek_v41")
    assert [(c.name, c.arguments) for c in p.calls] == [("get_weather", {"city": "Berlin", "days": 2})]


def test_headless_call_inferred_from_parameters():
    text = 'ok <parameter name="query">tcgen05</parameter><parameter name="limit">5</parameter></invoke>'
    p = _check(text, "deepseek_v41")
    assert p.content == "ok"
    assert [(c.name, c.arguments) for c in p.calls] == [("search", {"query": "tcgen05", "limit": 5})]


def test_headless_ambiguous_or_missing_required_stays_text():
    both = TOOLS + [{"type": "function", "function": {"name": "lookup", "parameters": {
        "type": "object", "properties": {"query": {"type": "string"}}, "required": ["query"]}}}]
    text = '<parameter name="query">x</parameter></invoke>'
    assert _check(text, "deepseek_v41", both).calls == []  # search and lookup both cover {query}
    text2 = '<parameter name="limit">3</parameter></invoke>'  # search covers it but misses "query"
    p = _check(text2, "deepseek_v41")
    assert p.calls == [] and p.content == text2


def test_candidate_with_prose_outside_values_is_restored():
    text = '<invoke name="get_weather">I think <parameter name="city">Oslo</parameter></invoke>'
    p = _check(text, "deepseek_v41")
    # the invoke is broken by prose; the parameter run after it is a headless call of get_weather
    assert "I think" in p.content and '<invoke name="get_weather">' in p.content
    assert [(c.name, c.arguments) for c in p.calls] == [("get_weather", {"city": "Oslo"})]


def test_unclosed_candidate_at_end_is_text():
    text = 'a <invoke name="get_weather"><parameter name="city">Oslo</parameter>'
    p = _check(text, "deepseek_v41")
    assert p.calls == [] and p.content == text


def test_no_recovery_inside_thinking_or_code_fence():
    call = '<invoke name="get_weather"><parameter name="city">Oslo</parameter></invoke>'
    p = _check(f"<think>maybe {call}</think>fine", "deepseek_v41")
    assert p.calls == [] and call in p.reasoning and p.content == "fine"
    fenced = f"Example:\n```\n{call}\n```\nend"
    p = _check(fenced, "deepseek_v41")
    assert p.calls == [] and call in p.content
    after = f"```\ncode\n```\n{call}"
    assert len(_check(after, "deepseek_v41").calls) == 1


def test_tool_choice_none_or_no_tools_recovers_nothing():
    call = _dsml_call("get_weather", [("city", "Oslo", "true")])
    for tools, choice in ((TOOLS, "none"), (None, "auto")):
        p = _check(call, "deepseek_v41", tools, choice)
        assert p.calls == [] and p.content == call


def test_stream_never_leaks_held_markup():
    text = "Hi " + _dsml_call("get_weather", [("city", "Oslo", "true")]) + " bye"
    sp = P.StreamParser("deepseek_v41", TOOLS)
    seen = ""
    for ch in text:
        _, c, _ = sp.feed(ch)
        seen += c
        assert "DSML" not in seen and "<｜" not in seen
    _, c, calls = sp.finish()
    assert (seen + c).strip() == "Hi  bye"
    assert len(sp.calls) == 1


def test_generic_family_unchanged():
    calls, content = P.parse_tool_calls('hi <tool_call>{"name": "f", "arguments": {"a": 1}}</tool_call>')
    assert calls[0].name == "f" and calls[0].arguments == {"a": 1} and content == "hi"
    p = _check("<tool_call>{'name': 'g', 'arguments': {'x': 2,},}</tool_call>", "generic", None)
    assert p.calls[0].arguments == {"x": 2}
