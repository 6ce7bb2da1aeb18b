"""Prompt datasets with score history and adaptive sampling.

Reference: ``BaseDataset.sample`` and the dataset registry (``axrl/datasets/base_dataset.py:148-175``,
``axrl/datasets/__init__.py:14-43``).  Sample types: ``uniform``, ``uniform-no-easy`` (skip prompts
whose recent success rate is >= 90 %), ``low-success-rate`` and ``intermediate-success-rate``
(weight prompts by how much signal their recent groups carry).
"""

from __future__ import annotations

from collections import defaultdict, deque
from typing import Callable

import numpy as np

from axrl_b200.data.conversation import Conversation, Message

_REGISTRY: dict[str, Callable[..., "BaseDataset"]] = {}


def register_dataset(name: str) -> Callable:
    def deco(cls):  # noqa: ANN001, ANN202
        _REGISTRY[name] = cls
        return cls

    return deco


def get_dataset(name: str, **kw) -> "BaseDataset":  # noqa: ANN003
    if name not in _REGISTRY:
        raise KeyError(f"unknown dataset {name!r}; registered: {sorted(_REGISTRY)}")
    return _REGISTRY[name](**kw)


class BaseDataset:
    def __init__(self, conversations: list[Conversation] | None = None, history_size: int = 64, seed: int = 0) -> None:
        self.conversations = conversations or []
        self.history: dict[str, deque] = defaultdict(lambda: deque(maxlen=history_size))
        self.length_history: dict[str, deque] = defaultdict(lambda: deque(maxlen=history_size))
        self.rng = np.random.default_rng(seed)

    def initialize(self) -> None:
        pass

    def __len__(self) -> int:
        return len(self.conversations)

    def update_score_history(self, conversation_id: str, scores: list[float]) -> None:
        self.history[conversation_id].extend(scores)

    def update_length_history(self, conversation_id: str, lengths: list[int]) -> None:
        self.length_history[conversation_id].extend(lengths)

    def success_rate(self, cid: str) -> float | None:
        h = self.history.get(cid)
        return float(np.mean(h)) if h else None

    def sample(self, n: int, sample_type: str = "uniform", epsilon: float = 0.05, sort_by_length: bool = False) -> list[Conversation]:
        N = len(self.conversations)
        assert N > 0, "empty dataset"
        w = np.ones(N)
        for i, c in enumerate(self.conversations):
            sr = self.success_rate(c.conversation_id)
            if sr is None:
                continue
            if sample_type == "uniform-no-easy" and sr >= 0.9:
                w[i] = 0.0
            elif sample_type == "low-success-rate":
                w[i] = (1.0 - sr) + epsilon
            elif sample_type == "intermediate-success-rate":
                w[i] = sr * (1.0 - sr) + epsilon
        if w.sum() <= 0:
            w = np.ones(N)
        idx = self.rng.choice(N, size=n, replace=n > N, p=w / w.sum())
        out = [self.conversations[i].deep_copy() for i in idx]
        if sort_by_length:
            out.sort(key=lambda c: -float(np.mean(self.length_history.get(c.conversation_id) or [0])))
        return out

    def state_dict(self) -> dict:
        return {"history": {k: list(v) for k, v in self.history.items()}, "length_history": {k: list(v) for k, v in self.length_history.items()}}

    def load_state_dict(self, sd: dict) -> None:
        for k, v in sd.get("history", {}).items():
            self.history[k].extend(v)
        for k, v in sd.get("length_history", {}).items():
            self.length_history[k].extend(v)


@register_dataset("synthetic_tokens")
class SyntheticTokenDataset(BaseDataset):
    """Prompts of uniform-random token ids (benchmark / plumbing workloads)."""

    def __init__(self, num: int = 256, prompt_len: int = 512, vocab_size: int = 151936, seed: int = 0, **kw) -> None:  # noqa: ANN003
        super().__init__(seed=seed, **kw)
        self.prompt_len, self.vocab_size = prompt_len, vocab_size
        rng = np.random.default_rng(seed)
        for i in range(num):
            c = Conversation(messages=[Message("user", "")], conversation_id=f"syn-{i}")
            c.gen_state.input_ids = rng.integers(1, vocab_size, size=prompt_len).astype(np.int32)
            c.extra["answer_token"] = 7
            self.conversations.append(c)


@register_dataset("parquet_qa")
class ParquetQADataset(BaseDataset):
    """Question/answer parquet (GSM8K, DAPO-17k, AIME style): columns ``question``/``prompt`` and ``answer``."""

    def __init__(self, path: str, question_key: str = "question", answer_key: str = "answer", limit: int | None = None, **kw) -> None:  # noqa: ANN003
        super().__init__(**kw)
        import pandas as pd

        df = pd.read_parquet(path)
        if limit:
            df = df.head(limit)
        for i, row in enumerate(df.itertuples(index=False)):
            d = row._asdict()
            q = d.get(question_key) or d.get("prompt")
            c = Conversation(messages=[Message("user", str(q))], conversation_id=f"{path}:{i}", extra={"answer": str(d.get(answer_key))})
            self.conversations.append(c)
