"""Search-R1: multi-turn tool-use RL where the model searches a corpus before answering.

Reference: ``axis_recipe/search_r1/search_env.py:41-266`` (retrieval server + FAISS, tool tags,
exact-match reward).  The model writes ``<search>query</search>`` to call the retriever; the
environment appends ``<information>...</information>`` (not trained) and the model continues; an
``<answer>...</answer>`` ends the episode.  Reward: normalised exact match with any gold answer.

Retrieval: :class:`BM25Index` (in process) or :class:`RetrievalClient` against a service speaking
``POST /retrieve {"queries": [...], "topk": k} -> {"result": [[{"contents": ...}, ...], ...]}``
(the interface of the reference's retrieval server); :func:`create_retrieval_app` serves an index.
"""

from __future__ import annotations

import math
import re
import string
from collections import Counter
from typing import Any

import numpy as np

from axrl_b200.data.conversation import GenerationInput, RolloutResult
from axrl_b200.data.rollout_trace import RolloutTrace
from axrl_b200.metrics.response_metric import ResponseMetric
from axrl_b200.processor.tokenizer import ChatTokenizer
from axrl_b200.recipe.base_recipe import BaseRecipe

SEARCH_PROMPT = ("Answer the question. You may search the knowledge base by writing <search> query </search>; results are "
                 "returned between <information> and </information>. When you know the answer, write <answer> answer </answer>.")
_WORD = re.compile(r"\w+")


class BM25Index:
    def __init__(self, docs: list[str], k1: float = 1.5, b: float = 0.75) -> None:
        self.docs = docs
        self.tf = [Counter(_WORD.findall(d.lower())) for d in docs]
        self.len = np.array([sum(t.values()) for t in self.tf], dtype=np.float64)
        self.avg = float(self.len.mean()) if len(docs) else 0.0
        df = Counter(w for t in self.tf for w in t)
        n = len(docs)
        self.idf = {w: math.log(1 + (n - c + 0.5) / (c + 0.5)) for w, c in df.items()}
        self.k1, self.b = k1, b

    def search(self, query: str, topk: int = 3) -> list[str]:
        q = _WORD.findall(query.lower())
        scores = np.zeros(len(self.docs))
        for i, tf in enumerate(self.tf):
            norm = self.k1 * (1 - self.b + self.b * self.len[i] / max(self.avg, 1e-9))
            scores[i] = sum(self.idf.get(w, 0.0) * tf[w] * (self.k1 + 1) / (tf[w] + norm) for w in q if w in tf)
        order = np.argsort(-scores, kind="stable")[:topk]
        return [self.docs[i] for i in order if scores[i] > 0]


class RetrievalClient:
    def __init__(self, url: str, timeout_s: float = 30.0) -> None:
        self.url, self.timeout_s = url.rstrip("/"), timeout_s

    def search(self, query: str, topk: int = 3) -> list[str]:
        import requests

        r = requests.post(self.url + "/retrieve", json={"queries": [query], "topk": topk}, timeout=self.timeout_s)
        r.raise_for_status()
        return [d["contents"] for d in r.json()["result"][0]]


def create_retrieval_app(index: BM25Index):  # noqa: ANN201
    from fastapi import FastAPI

    app = FastAPI()

    @app.post("/retrieve")
    async def retrieve(body: dict) -> dict:
        k = int(body.get("topk", 3))
        return {"result": [[{"contents": d} for d in index.search(q, k)] for q in body["queries"]]}

    return app


def normalize_answer(s: str) -> str:
    s = s.lower()
    s = "".join(ch for ch in s if ch not in set(string.punctuation))
    s = re.sub(r"\b(a|an|the)\b", " ", s)
    return " ".join(s.split())


def exact_match(pred: str | None, golds: list[str]) -> float:
    if pred is None:
        return 0.0
    p = normalize_answer(pred)
    return 1.0 if any(p == normalize_answer(g) for g in golds) else 0.0


def parse_action(text: str) -> tuple[str, str | None]:
    """('answer', a) | ('search', q) | ('none', None) from the latest tags in ``text``."""
    a = re.findall(r"<answer>(.*?)</answer>", text, re.S)
    if a:
        return "answer", a[-1].strip()
    q = re.findall(r"<search>(.*?)</search>", text, re.S)
    if q:
        return "search", q[-1].strip()
    return "none", None


class SearchR1Recipe(BaseRecipe):
    def __init__(self, config: Any, tokenizer: Any, dataset: Any, retriever: Any, max_turns: int = 4, topk: int = 3,
                 test: Any = None) -> None:
        super().__init__(config)
        self.tok = tokenizer if isinstance(tokenizer, ChatTokenizer) else ChatTokenizer(tokenizer)
        self.dataset, self.test = dataset, test
        self.retriever, self.max_turns, self.topk = retriever, max_turns, topk
        for ds in (dataset, test):
            if ds is not None:
                for c in ds.conversations:
                    msgs = [{"role": "system", "content": SEARCH_PROMPT}] + [{"role": m.role, "content": m.text()} for m in c.messages]
                    c.gen_state.input_ids = np.asarray(self.tok.render(msgs), dtype=np.int32)

    def get_test_datasets(self) -> list[tuple[str, Any]]:
        return [("search_r1_test", self.test)] if self.test is not None else []

    async def run_rollout(self, conversation: Any, runtime: Any) -> RolloutResult:
        ids = np.asarray(conversation.gen_state.input_ids)
        sid = f"{conversation.extra.get('group_id', conversation.conversation_id)}#{conversation.extra.get('group_index', 0)}"
        trace = RolloutTrace(max_length=self.config.train_sampling_config.max_total_tokens)
        trace.initialize(ids)
        answer, searches, finish, resp_len = None, 0, "length", 0
        for _turn in range(self.max_turns):
            cur = trace.token_ids
            room = self.config.train_sampling_config.max_total_tokens - len(cur)
            if room <= 8:
                break
            out = await runtime.rollout_worker.generate(GenerationInput(session_id=sid, input_ids=cur, sampling_config=self.config.train_sampling_config))
            trace.append_assistant(out.output_ids, out.output_logprobs)
            resp_len += len(out.output_ids)
            finish = out.finish_reason
            kind, arg = parse_action(self.tok.decode(out.output_ids.tolist()))
            if kind == "answer":
                answer = arg
                break
            if kind != "search":
                break
            searches += 1
            docs = self.retriever.search(arg, self.topk)
            info = "<information>" + "\n".join(f"Doc {i + 1}: {d}" for i, d in enumerate(docs)) + "</information>"
            trace.append_user_or_tool_message(np.asarray(self.tok.append_message_ids("tool", info), dtype=np.int32), "tool_result")
        golds = conversation.extra.get("answers") or [conversation.extra.get("answer", "")]
        score = exact_match(answer, [str(g) for g in golds])
        metric = ResponseMetric(score=score, response_length=resp_len, prompt_length=len(ids), finish_reason=finish,
                                num_turns=searches + 1, extra={"num_searches": float(searches)})
        return RolloutResult(conversation=conversation, trace=trace, metric=metric)
