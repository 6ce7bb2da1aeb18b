"""Response metrics (diversity, n-gram repetition, reasoning cues, finish reasons, low-quality rule,
pos/neg and per-subset aggregation) and the single-turn math environment."""

import asyncio

import numpy as np

from axrl_b200.data.conversation import Conversation, GenerationOutput, Message, RolloutResult
from axrl_b200.metrics.response_metric import (ResponseMetric, ResponseMetricCalculator, aggregate_response_metrics,
                                               aggregate_response_metrics_by_subset, ngram_repetition)


def _out(ids, text="", reason="stop"):
    return GenerationOutput(session_id="s", output_ids=np.asarray(ids), output_logprobs=np.zeros(len(ids), np.float32), output_text=text,
                            output_text_with_special_tokens=text, cached_tokens=3, finish_reason=reason, e2e_elapsed_seconds=1.5,
                            stop_reason=None, retry=2)


def test_calculator_fields():
    text = "Wait, let me re-check this.\nBecause 2+2=4, therefore the answer is 4.\n" + "x" * 50
    m = ResponseMetricCalculator().process(_out([1, 2, 3, 1, 2, 3, 4], text, "length"), prompt_length=9, score=1.0)
    assert m.response_length == m.token_count == 7 and m.prompt_length == 9
    assert abs(m.token_unique_ratio - 4 / 7) < 1e-9
    assert m.word_length_max == 50 and m.line_length_max == 50
    assert m.reasoning_behavior_backtracking == 1.0 and m.reasoning_behavior_verification == 1.0 and m.reasoning_behavior_causal == 1.0
    assert (m.rollout_cached_tokens, m.rollout_num_retry, m.finish_reason) == (3, 2, "length")
    assert m.is_low_quality == 0.0
    d = m.to_dict()
    assert d["rollout_finish_reason_length"] == 1.0 and d["rollout_finish_reason_stop"] == 0.0


def test_ngram_repetition_and_low_quality():
    assert ngram_repetition(list(range(100)), n=20) == 0.0
    loop = [5, 6, 7, 8] * 1200  # 4800 tokens of a 4-token loop
    rep = ngram_repetition(loop, n=20)
    assert rep > 0.99
    m = ResponseMetricCalculator().process(_out(loop, "a b c"))
    assert m.is_low_quality == 1.0


def test_aggregation_pos_neg_and_subsets():
    ms = [ResponseMetric(score=1.0, response_length=10, finish_reason="stop"), ResponseMetric(score=0.0, response_length=30, finish_reason="length"),
          ResponseMetric(score=1.0, response_length=20, finish_reason="stop")]
    a = aggregate_response_metrics(ms, "P", 2.0)
    assert a["P/num"] == 3 and a["P/response_length_mean"] == 20.0
    assert a["P/token_count__pos"] == 15.0 and a["P/token_count__neg"] == 30.0 and a["P/rollout_number__all"] == 3
    assert a["P/token_count_max__all"] == 30 and a["P/throughput_tokens_per_second"] == 30.0
    assert abs(a["P/rollout_finish_reason_length__all"] - 1 / 3) < 1e-9
    res = [RolloutResult(Conversation(extra={"src": s}), None, m) for s, m in zip(["a", "b", "a"], ms)]
    sub = aggregate_response_metrics_by_subset(res, "src", "E")
    assert sub["E/a/num"] == 2 and sub["E/b/num"] == 1
    assert aggregate_response_metrics_by_subset(res[:1], "src", "E") == {}


def test_math_env_single_step():
    from axrl_b200.envs.math_env import MathEnv

    class Exact:
        def verify(self, text, label):
            return 1.0 if label in text else 0.0

    conv = Conversation(messages=[Message(role="user", content="1+1?")])
    conv.gen_state.input_ids = np.arange(5, dtype=np.int32)
    env = MathEnv(Exact(), conv, ["3", "2"], max_length=64)
    out = _out([7, 8, 9], "the answer is 2")
    obs, reward, done, trace, metric = asyncio.run(env.step(out))
    assert reward == 1.0 and done and metric.score == 1.0 and metric.prompt_length == 5
    assert obs.messages[-1].role == "assistant" and obs.messages[-1].text() == "the answer is 2"
    s = trace.to_sample()
    assert list(s.input_ids[:8]) == [0, 1, 2, 3, 4, 7, 8, 9]
    assert int(s.loss_mask.sum()) == 3
    env2 = MathEnv(Exact(), conv, "5", max_length=64, return_sample=False)
    _, r2, _, t2, _ = asyncio.run(env2.step(out))
    assert r2 == 0.0 and t2 is None
