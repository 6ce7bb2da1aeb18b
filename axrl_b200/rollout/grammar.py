"""Grammar-constrained decoding: regular expressions and a JSON-schema subset over token vocabularies.

Reference: the SGLang engines' ``json_schema`` / ``regex`` / ``structural_tag`` sampling
constraints, set from tool-call requests in ``axrl/worker/sglang_worker.py:192-244`` (xgrammar in
SGLang).  Here:

* :func:`compile_regex` parses a regular expression (literals, ``.``, classes with ranges and
  negation, the ``\\d \\w \\s`` escapes, groups, ``|``, ``* + ?`` and ``{m}``, ``{m,}``, ``{m,n}``)
  into a Thompson NFA over characters; DFA states (epsilon-closed NFA state sets) are built
  lazily.  Every Thompson state lies on a path to the accepting state, so a non-empty state set
  means "still a prefix of some match".
* :func:`schema_to_regex` turns a JSON schema (objects with properties / required, arrays with
  ``items`` / ``minItems``, strings, numbers, integers, booleans, null, ``enum``, ``const``,
  ``anyOf`` / ``oneOf``) into such an expression; whitespace between tokens is an optional single
  space, the layout tool-call JSON uses.
* :class:`TokenGrammar` lifts the character automaton to token ids: the tokens allowed in a state
  are found by walking a trie of the vocabulary's token strings with the automaton (pruned as soon
  as a prefix dies), cached per state; end-of-sequence is allowed in accepting states.

The rollout engine applies the allowed set of each constrained row as an additive ``-inf`` bias
before sampling and advances the row's state with the sampled token.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np

# ----------------------------------------------------------------------------- regex -> NFA

_ANY = ("any",)


def _cls_match(cls: tuple, ch: str) -> bool:
    if cls is _ANY:
        return ch != "\n"
    neg, chars, ranges = cls
    hit = ch in chars or any(a <= ch <= b for a, b in ranges)
    return hit != neg


_ESC = {"d": (False, frozenset(), (("0", "9"),)), "w": (False, frozenset("_"), (("a", "z"), ("A", "Z"), ("0", "9"))),
        "s": (False, frozenset(" \t\n\r\f\v"), ())}
_ESC.update({k.upper(): (True, v[1], v[2]) for k, v in list(_ESC.items())})


class _Parser:
    def __init__(self, pattern: str) -> None:
        self.p, self.i = pattern, 0

    def peek(self) -> str | None:
        return self.p[self.i] if self.i < len(self.p) else None

    def take(self) -> str:
        c = self.p[self.i]
        self.i += 1
        return c

    def parse(self):  # noqa: ANN201
        node = self.alt()
        if self.i != len(self.p):
            raise ValueError(f"unexpected {self.p[self.i]!r} at {self.i} in regex")
        return node

    def alt(self):  # noqa: ANN201
        branches = [self.seq()]
        while self.peek() == "|":
            self.take()
            branches.append(self.seq())
        return ("alt", branches) if len(branches) > 1 else branches[0]

    def seq(self):  # noqa: ANN201
        items = []
        while self.peek() is not None and self.peek() not in "|)":
            items.append(self.quant(self.atom()))
        return ("seq", items)

    def quant(self, node):  # noqa: ANN001, ANN201
        while True:
            c = self.peek()
            if c == "*":
                self.take()
                node = ("rep", node, 0, None)
            elif c == "+":
                self.take()
                node = ("rep", node, 1, None)
            elif c == "?":
                self.take()
                node = ("rep", node, 0, 1)
            elif c == "{":
                j = self.p.find("}", self.i)
                body = self.p[self.i + 1:j]
                if j < 0 or not body.replace(",", "").isdigit() and body != "":
                    return node  # a literal '{'
                self.i = j + 1
                if "," in body:
                    a, b = body.split(",", 1)
                    node = ("rep", node, int(a or 0), int(b) if b else None)
                else:
                    node = ("rep", node, int(body), int(body))
            else:
                return node

    def atom(self):  # noqa: ANN201
        c = self.take()
        if c == "(":
            if self.p.startswith("?:", self.i):
                self.i += 2
            node = self.alt()
            if self.peek() != ")":
                raise ValueError("unbalanced parenthesis in regex")
            self.take()
            return node
        if c == "[":
            return ("cls", self.cls())
        if c == ".":
            return ("cls", _ANY)
        if c == "\\":
            e = self.take()
            if e in _ESC:
                return ("cls", _ESC[e])
            return ("cls", (False, frozenset({{"n": "\n", "t": "\t", "r": "\r"}.get(e, e)}), ()))
        return ("cls", (False, frozenset(c), ()))

    def cls(self) -> tuple:
        neg = self.peek() == "^"
        if neg:
            self.take()
        chars, ranges, first = set(), [], True
        while True:
            c = self.take()
            if c == "]" and not first:
                break
            first = False
            if c == "\\":
                e = self.take()
                if e in _ESC and not _ESC[e][0]:
                    chars |= _ESC[e][1]
                    ranges += list(_ESC[e][2])
                    continue
                c = {"n": "\n", "t": "\t", "r": "\r"}.get(e, e)
            if self.peek() == "-" and self.i + 1 < len(self.p) and self.p[self.i + 1] != "]":
                self.take()
                hi = self.take()
                if hi == "\\":
                    hi = self.take()
                ranges.append((c, hi))
            else:
                chars.add(c)
        return (neg, frozenset(chars), tuple(ranges))


@dataclass
class _NFA:
    eps: list[list[int]] = field(default_factory=list)
    edges: list[list[tuple[tuple, int]]] = field(default_factory=list)

    def new(self) -> int:
        self.eps.append([])
        self.edges.append([])
        return len(self.eps) - 1


def _build(nfa: _NFA, node) -> tuple[int, int]:  # noqa: ANN001
    kind = node[0]
    if kind == "cls":
        a, b = nfa.new(), nfa.new()
        nfa.edges[a].append((node[1], b))
        return a, b
    if kind == "seq":
        a = nfa.new()
        cur = a
        for it in node[1]:
            s, e = _build(nfa, it)
            nfa.eps[cur].append(s)
            cur = e
        return a, cur
    if kind == "alt":
        a, b = nfa.new(), nfa.new()
        for br in node[1]:
            s, e = _build(nfa, br)
            nfa.eps[a].append(s)
            nfa.eps[e].append(b)
        return a, b
    if kind == "rep":
        _, sub, lo, hi = node
        a = nfa.new()
        cur = a
        for _ in range(lo):
            s, e = _build(nfa, sub)
            nfa.eps[cur].append(s)
            cur = e
        end = nfa.new()
        if hi is None:  # loop
            s, e = _build(nfa, sub)
            nfa.eps[cur].append(s)
            nfa.eps[e].append(s)
            nfa.eps[e].append(end)
            nfa.eps[cur].append(end)
        else:
            for _ in range(hi - lo):
                s, e = _build(nfa, sub)
                nfa.eps[cur].append(s)
                nfa.eps[cur].append(end)
                cur = e
            nfa.eps[cur].append(end)
        return a, end
    raise ValueError(kind)


class CharDFA:
    """Lazily determinised automaton; states are small ints, -1 is the dead state."""

    def __init__(self, pattern: str) -> None:
        self.nfa = _NFA()
        self.start_nfa, self.accept_nfa = _build(self.nfa, _Parser(pattern).parse())
        self.sets: list[frozenset] = []
        self.index: dict[frozenset, int] = {}
        self.trans: list[dict[str, int]] = []
        self.start = self._state(self._closure({self.start_nfa}))

    def _closure(self, states) -> frozenset:  # noqa: ANN001
        stack, seen = list(states), set(states)
        while stack:
            s = stack.pop()
            for t in self.nfa.eps[s]:
                if t not in seen:
                    seen.add(t)
                    stack.append(t)
        return frozenset(seen)

    def _state(self, st: frozenset) -> int:
        if not st:
            return -1
        i = self.index.get(st)
        if i is None:
            i = len(self.sets)
            self.sets.append(st)
            self.index[st] = i
            self.trans.append({})
        return i

    def step(self, state: int, ch: str) -> int:
        if state < 0:
            return -1
        nxt = self.trans[state].get(ch)
        if nxt is None:
            moved = {t for s in self.sets[state] for cls, t in self.nfa.edges[s] if _cls_match(cls, ch)}
            nxt = self._state(self._closure(moved)) if moved else -1
            self.trans[state][ch] = nxt
        return nxt

    def walk(self, state: int, text: str) -> int:
        for ch in text:
            state = self.step(state, ch)
            if state < 0:
                return -1
        return state

    def accepting(self, state: int) -> bool:
        return state >= 0 and self.accept_nfa in self.sets[state]

    def fullmatch(self, text: str) -> bool:
        return self.accepting(self.walk(self.start, text))


def compile_regex(pattern: str) -> CharDFA:
    return CharDFA(pattern)


# ----------------------------------------------------------------------------- JSON schema -> regex

_WS = " ?"
_STR = r'"([^"\\]|\\["\\/bfnrt])*"'
_INT = r"-?(0|[1-9][0-9]*)"
_NUM = r"-?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][+-]?[0-9]+)?"
_META = set("\\.^$|?*+()[]{}")


def _lit(s: str) -> str:
    return "".join("\\" + c if c in _META else c for c in s)


def schema_to_regex(schema: Any) -> str:
    """Regular expression accepting the JSON texts (compact, optional single spaces) of ``schema``."""
    if isinstance(schema, str):
        schema = json.loads(schema)
    if schema is True or schema == {}:
        schema = {"type": ["string", "number", "boolean", "null"]}
    if "const" in schema:
        return _lit(json.dumps(schema["const"]))
    if "enum" in schema:
        return "(" + "|".join(_lit(json.dumps(v)) for v in schema["enum"]) + ")"
    for key in ("anyOf", "oneOf"):
        if key in schema:
            return "(" + "|".join(schema_to_regex(s) for s in schema[key]) + ")"
    t = schema.get("type")
    if isinstance(t, list):
        return "(" + "|".join(schema_to_regex({**schema, "type": x}) for x in t) + ")"
    if t == "string":
        return _STR
    if t == "integer":
        return _INT
    if t == "number":
        return _NUM
    if t == "boolean":
        return "(true|false)"
    if t == "null":
        return "null"
    if t == "array":
        item = schema_to_regex(schema.get("items", True))
        lo = int(schema.get("minItems", 0))
        more = f"({_WS},{_WS}{item})*"
        body = f"{item}{more}" if lo >= 1 else f"({item}{more})?"
        return rf"\[{_WS}{body}{_WS}\]"
    if t == "object" or "properties" in schema:
        props = list(schema.get("properties", {}).items())
        required = set(schema.get("required", [n for n, _ in props]))
        parts = [(f"{_lit(json.dumps(n))}{_WS}:{_WS}{schema_to_regex(sub)}", n in required) for n, sub in props]
        return _object(parts)
    raise ValueError(f"unsupported JSON schema: {schema}")


def _object(parts: list[tuple[str, bool]]) -> str:
    """Properties in declared order, optional ones may be left out: one alternative per choice of
    the first emitted property (every property before it must be optional)."""
    alts = []
    for i, (kv, req) in enumerate(parts):
        rest = "".join(f"{_WS},{_WS}{k}" if r else f"({_WS},{_WS}{k})?" for k, r in parts[i + 1:])
        alts.append(kv + rest)
        if req:
            break
    else:
        alts.append("")  # every property optional: the empty object too
    body = alts[0] if len(alts) == 1 else "(" + "|".join(alts) + ")"
    return rf"\{{{_WS}{body}{_WS}\}}"


# ----------------------------------------------------------------------------- token level


class _Trie:
    __slots__ = ("kids", "ids")

    def __init__(self) -> None:
        self.kids: dict[str, _Trie] = {}
        self.ids: list[int] = []


class TokenGrammar:
    """Allowed-token masks of a character automaton over a vocabulary of token strings."""

    def __init__(self, dfa: CharDFA, token_strings: Sequence[str], eos_ids: Sequence[int]) -> None:
        self.dfa = dfa
        self.V = len(token_strings)
        self.eos = [int(e) for e in eos_ids if 0 <= int(e) < self.V]
        self.strings = list(token_strings)
        self.root = _Trie()
        for i, s in enumerate(token_strings):
            if not s or i in self.eos:
                continue
            node = self.root
            for ch in s:
                node = node.kids.setdefault(ch, _Trie())
            node.ids.append(i)
        self.masks: dict[int, np.ndarray] = {}

    @property
    def start(self) -> int:
        return self.dfa.start

    def allowed(self, state: int) -> np.ndarray:
        m = self.masks.get(state)
        if m is not None:
            return m
        m = np.zeros(self.V, dtype=bool)
        if state >= 0:
            stack = [(self.root, state)]
            while stack:
                node, st = stack.pop()
                for ch, kid in node.kids.items():
                    nst = self.dfa.step(st, ch)
                    if nst < 0:
                        continue
                    if kid.ids:
                        m[kid.ids] = True
                    if kid.kids:
                        stack.append((kid, nst))
            if self.dfa.accepting(state):
                m[self.eos] = True
        if not m.any():  # no continuation (tokenisation cannot express the rest): let the row end
            m[self.eos] = True
        self.masks[state] = m
        return m

    def advance(self, state: int, token: int) -> int:
        if token in self.eos or not (0 <= token < self.V):
            return state
        return self.dfa.walk(state, self.strings[token])


def make_token_grammar(*, regex: str | None = None, json_schema: Any = None, token_strings: Sequence[str],
                       eos_ids: Sequence[int]) -> TokenGrammar:
    pattern = regex if regex is not None else schema_to_regex(json_schema)
    return TokenGrammar(compile_regex(pattern), token_strings, eos_ids)


def tool_call_schema(tools: Sequence[dict] | None, tool_choice: Any) -> dict | None:
    """JSON schema forcing a tool call, as the reference's SGLang worker builds it for
    ``tool_choice="required"`` or a named function (``axrl/worker/sglang_worker.py:199-209``): a
    non-empty list of ``{"name": <tool>, "parameters": <its schema>}`` objects.  None for ``"auto"``
    / ``"none"`` / no tools (unconstrained)."""
    if not tools or tool_choice in (None, "auto", "none"):
        return None
    fns = [t.get("function", t) for t in tools]
    if isinstance(tool_choice, dict):  # {"type": "function", "function": {"name": ...}}
        name = tool_choice.get("function", tool_choice).get("name")
        fns = [f for f in fns if f.get("name") == name]
        if not fns:
            raise ValueError(f"tool_choice names an unknown function: {name}")
    items = [{"type": "object", "properties": {"name": {"const": f["name"]},
                                               "parameters": f.get("parameters") or {"type": "object", "properties": {}}},
              "required": ["name", "parameters"]} for f in fns]
    return {"type": "array", "minItems": 1, "items": items[0] if len(items) == 1 else {"anyOf": items}}


class StructuralTagGrammar:
    """Free text in which every tagged segment is constrained (the reference's ``structural_tag``
    constraint for ``tool_choice="auto"``, ``axrl/worker/sglang_worker.py:211-238``): once the text
    ends with a trigger (e.g. ``<tool_call>``), the continuation must be one of the structures whose
    ``begin`` starts with that trigger, i.e. ``begin`` + JSON of ``schema`` + ``end``; after ``end``
    the text is free again.

    States are ints: -1 - k encodes free text whose last ``k`` characters may still start a trigger
    (a bounded suffix is kept in ``self.tails``); >= 0 are states of the tagged-segment automaton.
    If a token completes a trigger and continues with text the structure does not allow, the
    segment is left unconstrained (free) rather than rejected."""

    def __init__(self, structures: Sequence[dict], triggers: Sequence[str], token_strings: Sequence[str], eos_ids: Sequence[int]) -> None:
        self.triggers = list(triggers)
        self.strings = list(token_strings)
        self.V = len(token_strings)
        self.eos = [int(e) for e in eos_ids if 0 <= int(e) < self.V]
        alts: dict[str, list[str]] = {}
        for s in structures:
            trig = next((t for t in self.triggers if s["begin"].startswith(t)), None)
            if trig is None:
                raise ValueError(f"structure begin {s['begin']!r} does not start with a trigger")
            alts.setdefault(trig, []).append(_lit(s["begin"][len(trig):]) + schema_to_regex(s.get("schema", True)) + _lit(s["end"]))
        self.segment = {t: TokenGrammar(compile_regex("(" + "|".join(a) + ")"), token_strings, eos_ids) for t, a in alts.items()}
        self.keep = max(len(t) for t in self.triggers)
        self.tails: list[str] = [""]  # state -1 - i -> free text tail
        self._tail_id = {"": 0}
        self._seg_ids: dict[tuple[str, int], int] = {}
        self._seg_rev: list[tuple[str, int]] = []
        self.masks: dict[int, np.ndarray] = {}

    @property
    def start(self) -> int:
        return -1

    def _free(self, tail: str) -> int:
        tail = tail[-self.keep:]
        i = self._tail_id.get(tail)
        if i is None:
            i = len(self.tails)
            self.tails.append(tail)
            self._tail_id[tail] = i
        return -1 - i

    def _seg(self, trig: str, inner: int) -> int:
        key = (trig, inner)
        i = self._seg_ids.get(key)
        if i is None:
            i = len(self._seg_rev)
            self._seg_rev.append(key)
            self._seg_ids[key] = i
        return i

    def allowed(self, state: int) -> np.ndarray:
        m = self.masks.get(state)
        if m is None:
            if state < 0:  # free text: anything
                m = np.ones(self.V, dtype=bool)
            else:
                trig, inner = self._seg_rev[state]
                g = self.segment[trig]
                m = g.allowed(inner).copy()
                if g.dfa.accepting(inner):  # segment complete: free text continues
                    m[:] = True
            self.masks[state] = m
        return m

    def advance(self, state: int, token: int) -> int:
        if token in self.eos or not (0 <= token < self.V):
            return state
        text = self.strings[token]
        if state >= 0:
            trig, inner = self._seg_rev[state]
            g = self.segment[trig]
            if g.dfa.accepting(inner):
                return self.advance(self._free(""), token)
            nxt = g.dfa.walk(inner, text)
            return self._seg(trig, nxt) if nxt >= 0 else self._free(text)
        buf = self.tails[-1 - state] + text
        for trig in self.triggers:
            j = buf.find(trig)
            if j >= 0 and trig in self.segment:
                g = self.segment[trig]
                inner = g.dfa.walk(g.dfa.start, buf[j + len(trig):])
                return self._seg(trig, inner) if inner >= 0 else self._free(buf[j + len(trig):])
        return self._free(buf)


def tool_call_structural_tag(tools: Sequence[dict] | None, tool_call_parser: str | None) -> dict | None:
    """Structural tag for ``tool_choice="auto"`` with the Qwen tool-call format (``<tool_call>`` JSON
    ``</tool_call>``, parsers "qwen" / "qwen25" / "qwen3"): one structure per tool whose arguments
    follow the tool's parameter schema."""
    if not tools or tool_call_parser not in ("qwen", "qwen25", "qwen3", "hermes"):
        return None
    structures = []
    for t in tools:
        f = t.get("function", t)
        structures.append({"begin": '<tool_call>\n{"name": ' + json.dumps(f["name"]) + ', "arguments": ',
                           "schema": f.get("parameters") or {"type": "object", "properties": {}}, "end": "}\n</tool_call>"})
    return {"type": "structural_tag", "structures": structures, "triggers": ["<tool_call>"]}
