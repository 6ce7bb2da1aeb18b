"""Single-turn math environment (reference ``axrl/envs/math_env.py:18-62``).

One ``step`` scores the model's answer with a verifier, computes the response metrics and records
the turn as a :class:`RolloutTrace` (prompt tokens + the generated tokens with their sampled
log-probabilities), then ends the episode.  The scorer, metric calculator and tokenizer are
injected, so the same environment serves GSM8K, MATH / DAPO or any verifier with
``verify(response_text, label) -> float`` (a synchronous verifier, or an async worker with
``generate``).
"""

from __future__ import annotations

import inspect
import logging
from typing import Any

import numpy as np

from axrl_b200.data.conversation import Conversation, GenerationOutput, Message
from axrl_b200.data.rollout_trace import RolloutTrace
from axrl_b200.envs.base_env import BaseEnv
from axrl_b200.metrics.response_metric import ResponseMetric, ResponseMetricCalculator

logger = logging.getLogger(__name__)


async def _call(worker: Any, method: str, *args: Any) -> Any:
    out = getattr(worker, method)(*args)
    return await out if inspect.isawaitable(out) else out


class MathEnv(BaseEnv):
    def __init__(self, score_provider: Any, conv: Conversation, label: str | list[str], *, max_length: int,
                 return_sample: bool = True, metric_calculator: Any = None, decode: Any = None) -> None:
        """``score_provider``: ``verify(text, label)`` (or an async ``generate`` worker taking
        ``(text, label)``); ``conv.gen_state.input_ids`` must hold the rendered prompt tokens;
        ``decode`` turns ids into text when the generation output carries none."""
        super().__init__(conv)
        assert self.conv.gen_state.input_ids is not None, "the prompt must be tokenised before the episode starts"
        self.score_provider = score_provider
        self.metric_calculator = metric_calculator or ResponseMetricCalculator()
        self.label = label
        self.max_length = max_length
        self.return_sample = return_sample
        self.decode = decode

    async def _score(self, text: str) -> float:
        labels = self.label if isinstance(self.label, list) else [self.label]
        best = 0.0
        for lab in labels:  # several accepted answers: the best match counts
            if hasattr(self.score_provider, "verify"):
                s = await _call(self.score_provider, "verify", text, lab)
            else:
                s = await _call(self.score_provider, "generate", text, lab)
            best = max(best, float(getattr(s, "score", s)))
        return best

    async def step(self, action: GenerationOutput) -> tuple[Conversation, float, bool, RolloutTrace | None, ResponseMetric]:
        """(observation, reward, done, trace or None, metric); always done after one step."""
        ids = np.asarray(action.output_ids)
        lps = np.asarray(action.output_logprobs)
        assert len(lps) == len(ids), "every generated token needs its sampled log-probability"
        text = action.output_text or (self.decode(ids.tolist()) if self.decode else "")
        score = await self._score(text)
        metric = await _call(self.metric_calculator, "generate", action) if hasattr(self.metric_calculator, "generate") \
            else self.metric_calculator.process(action)
        metric.score = score
        metric.prompt_length = len(self.conv.gen_state.input_ids)
        trace = RolloutTrace(max_length=self.max_length)
        trace.initialize(self.conv.gen_state.input_ids)
        trace.append_assistant_message(action)
        self.conv.add_message(Message(role="assistant", content=text))
        return self.conv, score, True, trace if self.return_sample else None, metric
