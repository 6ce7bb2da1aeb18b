"""Recipe over synthetic token prompts: one assistant turn, reward = token presence.

Used by the controller tests and as the smallest end-to-end example of the recipe API
(the GSM8K recipe of the reference, ``axis_recipe/grpo_gsm8k/train_pipeline.py:25-71``,
has the same shape with a tokenizer and a math verifier in place of the token rule).
"""

from __future__ import annotations

import numpy as np

from axrl_b200.data.conversation import GenerationInput, RolloutResult
from axrl_b200.data.rollout_trace import RolloutTrace
from axrl_b200.datasets.base_dataset import SyntheticTokenDataset
from axrl_b200.metrics.response_metric import ResponseMetric
from axrl_b200.recipe.base_recipe import BaseRecipe
from axrl_b200.verifier.token_presence import token_presence_reward


class SyntheticTokenRecipe(BaseRecipe):
    def __init__(self, config, num_prompts: int = 16, prompt_len: int = 32, vocab_size: int = 1024, reward_token: int = 7) -> None:  # noqa: ANN001
        super().__init__(config)
        self.dataset = SyntheticTokenDataset(num=num_prompts, prompt_len=prompt_len, vocab_size=vocab_size)
        self.reward_token = reward_token

    async def run_rollout(self, conversation, runtime) -> RolloutResult:  # noqa: ANN001
        ids = np.asarray(conversation.gen_state.input_ids)
        sid = f"{conversation.extra.get('group_id', conversation.conversation_id)}#{conversation.extra.get('group_index', 0)}"
        out = await runtime.rollout_worker.generate(GenerationInput(session_id=sid, input_ids=ids, sampling_config=self.config.train_sampling_config))
        trace = RolloutTrace(max_length=len(ids) + len(out.output_ids) + 1)
        trace.initialize(ids)
        trace.append_assistant(out.output_ids, out.output_logprobs)
        score = token_presence_reward(out.output_ids.tolist(), self.reward_token)
        metric = ResponseMetric(score=score, response_length=len(out.output_ids), prompt_length=len(ids), finish_reason=out.finish_reason,
                                repetition_ratio=ResponseMetric.repetition(out.output_ids.tolist()))
        return RolloutResult(conversation=conversation, trace=trace, metric=metric)

    def get_test_datasets(self) -> list[tuple[str, SyntheticTokenDataset]]:
        if not hasattr(self, "_test"):
            self._test = SyntheticTokenDataset(num=4, prompt_len=self.dataset.prompt_len, vocab_size=self.dataset.vocab_size, seed=99)
        return [("synthetic_test", self._test)]

    def build_sft_samples(self, dataset) -> list:  # noqa: ANN001
        """Target: the reward token repeated, then the prompt's first tokens (a learnable mapping)."""
        from axrl_b200.data.sample import Sample

        out = []
        for c in dataset.conversations:
            p = [int(t) for t in c.gen_state.input_ids]
            out.append(Sample.from_tokens(p, [self.reward_token] * 4 + p[:4]))
        return out
