"""Grammar-constrained decoding: regex / JSON-schema automata, token masks, and the rollout engine
producing only matching responses (tool-call JSON as the reference's SGLang worker constrains it,
``axrl/worker/sglang_worker.py:192-244``)."""

import json

from axrl_b200.rollout.grammar import compile_regex, make_token_grammar, schema_to_regex, tool_call_schema


def test_regex_automaton():
    d = compile_regex(r"(ab|cd)*x{2,3}[0-9]+(\.[a-f]?)?")
    for t in ("xx1", "abcdxxx42", "xx0.", "xx7.e"):
        assert d.fullmatch(t), t
    for t in ("x1", "abx", "xxxx1", "xx1.g", ""):
        assert not d.fullmatch(t), t
    assert compile_regex(r"[^\"\\]+").fullmatch("abc") and not compile_regex(r"[^\"\\]+").fullmatch('a"')
    assert compile_regex(r"\d{3}-\w+\s?").fullmatch("123-ab_9 ")


def test_json_schema_subset():
    sch = {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "boolean"},
                                            "c": {"type": "array", "items": {"enum": ["x", "y", 3]}}}, "required": ["b"]}
    d = compile_regex(schema_to_regex(sch))
    good = ['{"b": true}', '{"a": -3, "b": false}', '{"b": true, "c": ["x", 3]}', '{"a":0,"b":true,"c":[]}']
    for t in good:
        assert d.fullmatch(t), t
        json.loads(t)
    for t in ['{"a": 1}', '{"b": 1}', '{"b": true, "c": ["z"]}', '{"a": 01, "b": true}']:
        assert not d.fullmatch(t), t


def test_tool_call_schema_matches_reference_shape():
    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {
        "type": "object", "properties": {"city": {"type": "string"}}, "required": ["city"]}}},
             {"type": "function", "function": {"name": "search", "parameters": {
                 "type": "object", "properties": {"q": {"type": "string"}}, "required": ["q"]}}}]
    assert tool_call_schema(tools, "auto") is None and tool_call_schema(None, "required") is None
    d = compile_regex(schema_to_regex(tool_call_schema(tools, "required")))
    assert d.fullmatch('[{"name": "search", "parameters": {"q": "b200"}}]')
    d2 = compile_regex(schema_to_regex(tool_call_schema(tools, {"type": "function", "function": {"name": "get_weather"}})))
    assert d2.fullmatch('[{"name": "get_weather", "parameters": {"city": "Paris"}}]')
    assert not d2.fullmatch('[{"name": "search", "parameters": {"q": "b200"}}]')


def test_token_masks_follow_the_automaton():
    vocab = [chr(i) for i in range(32, 127)] + ['"get_weather"', '{"name": ', "<eos>"]
    eos = len(vocab) - 1
    g = make_token_grammar(regex=r'\{"name": "get_weather"\}', token_strings=vocab, eos_ids=[eos])
    st = g.start
    allowed = {vocab[i] for i in range(len(vocab)) if g.allowed(st)[i]}
    assert allowed == {"{", '{"name": '}
    for t in ('{"name": ', '"get_weather"', "}"):
        st = g.advance(st, vocab.index(t))
    m = g.allowed(st)
    assert m[eos] and m.sum() == 1  # complete: only end-of-sequence


class _CharTok:
    """Byte-level test tokenizer: id i < 256 is the character chr(i)."""

    def __init__(self, n: int) -> None:
        self.n = n

    def __len__(self) -> int:
        return self.n

    def decode(self, ids):  # noqa: ANN001, ANN201
        return "".join(chr(i) if 32 <= i < 127 else "" for i in ids)


def test_engine_generates_only_schema_conforming_json():
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16)
    m = Qwen3Model(cfg)
    m.init_weights(0)
    eos = 0
    eng = RolloutEngine(m, max_batch=4, kv_tokens=4096, max_context=512, use_cuda_graph=False, eos_token_id=eos,
                        tokenizer=_CharTok(256), burst=8)
    schema = {"type": "object", "properties": {"ok": {"type": "boolean"}, "n": {"type": "integer"}}, "required": ["ok", "n"]}
    reqs = [GenRequest(rid=f"r{i}", prompt=[65 + i, 66, 67], max_new_tokens=60, temperature=1.0, stop_token_ids=(eos,),
                       json_schema=schema) for i in range(3)]
    reqs.append(GenRequest(rid="plain", prompt=[70, 71], max_new_tokens=10, temperature=1.0))
    res = {r.rid: r for r in eng.generate(reqs)}
    d = compile_regex(schema_to_regex(schema))
    for i in range(3):
        r = res[f"r{i}"]
        text = "".join(chr(t) for t in r.output_ids if t != eos)
        if r.finish_reason == "stop":
            assert d.fullmatch(text), text
            json.loads(text)
        else:  # cut by max_new_tokens: still a valid prefix
            assert d.walk(d.start, text) >= 0, text
    assert sum(res[f"r{i}"].finish_reason == "stop" for i in range(3)) >= 2  # complete JSON documents
    assert len(res["plain"].output_ids) == 10


def test_structural_tag_constrains_only_tagged_segments():
    from axrl_b200.rollout.grammar import StructuralTagGrammar, tool_call_structural_tag

    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {
        "type": "object", "properties": {"city": {"type": "string"}}, "required": ["city"]}}}]
    tag = tool_call_structural_tag(tools, "qwen3")
    assert tag["triggers"] == ["<tool_call>"] and tool_call_structural_tag(tools, None) is None
    vocab = [chr(i) for i in range(32, 127)] + ["<tool_call>", "\n", "<eos>"]
    eos = len(vocab) - 1
    g = StructuralTagGrammar(tag["structures"], tag["triggers"], vocab, [eos])
    s = g.start
    for ch in "Sure.":
        assert g.allowed(s).all()
        s = g.advance(s, vocab.index(ch))
    s = g.advance(s, vocab.index("<tool_call>"))
    assert [vocab[i] for i in range(len(vocab)) if g.allowed(s)[i]] == ["\n"]
    body = '\n{"name": "get_weather", "arguments": {"city": "Oslo"}}\n</tool_call>'
    for ch in body:
        tok = vocab.index(ch) if ch != "\n" else vocab.index("\n")
        assert g.allowed(s)[tok], (ch, s)
        s = g.advance(s, tok)
    assert g.allowed(s).all()  # free text again after the end tag
