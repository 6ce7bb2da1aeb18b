"""GSM8K GRPO / PPO recipe.

Reference: ``axis_recipe/grpo_gsm8k/train_pipeline.py:25-71``: prompts from the GSM8K parquet
files rendered with the model's chat template, one assistant turn, reward from the GSM8K verifier
(last ``#### number``), GRPO by default or PPO with a value model.

Usage: ``PipelineController(cfg, Gsm8kRecipe(cfg, train_path=..., test_path=..., tokenizer=...))``.
"""

from __future__ import annotations

from typing import Any

import numpy as np

from axrl_b200.data.conversation import GenerationInput, RolloutResult
from axrl_b200.datasets.base_dataset import BaseDataset, ParquetQADataset
from axrl_b200.envs.math_env import MathEnv
from axrl_b200.processor.tokenizer import ChatTokenizer
from axrl_b200.recipe.base_recipe import BaseRecipe
from axrl_b200.verifier.gsm8k import compute_score

SYSTEM_PROMPT = "Solve the problem step by step. Put the final numeric answer after '####'."


class SingleTurnQARecipe(BaseRecipe):
    """One assistant turn scored by ``score(response_text, answer)``."""

    def __init__(self, config: Any, tokenizer: Any, train: BaseDataset, test: BaseDataset | None = None,
                 system_prompt: str | None = SYSTEM_PROMPT) -> None:
        super().__init__(config)
        self.tok = tokenizer if isinstance(tokenizer, ChatTokenizer) else ChatTokenizer(tokenizer)
        self.dataset, self.test = train, test
        self.system_prompt = system_prompt
        for ds in (train, test):
            if ds is not None:
                for c in ds.conversations:
                    self.tokenize(c)

    def score(self, text: str, answer: str) -> float:
        raise NotImplementedError

    def tokenize(self, conv: Any) -> None:
        msgs = ([{"role": "system", "content": self.system_prompt}] if self.system_prompt else [])
        msgs += [{"role": m.role, "content": m.text()} for m in conv.messages]
        conv.gen_state.input_ids = np.asarray(self.tok.render(msgs), dtype=np.int32)

    def get_test_datasets(self) -> list[tuple[str, BaseDataset]]:
        return [(type(self).__name__.replace("Recipe", "").lower() + "_test", self.test)] if self.test is not None else []

    def verify(self, text: str, answer: str) -> float:
        """Scorer interface of :class:`MathEnv`."""
        return self.score(text, answer)

    async def run_rollout(self, conversation: Any, runtime: Any) -> RolloutResult:
        ids = np.asarray(conversation.gen_state.input_ids)
        sid = f"{conversation.extra.get('group_id', conversation.conversation_id)}#{conversation.extra.get('group_index', 0)}"
        out = await runtime.rollout_worker.generate(GenerationInput(session_id=sid, input_ids=ids, sampling_config=self.config.train_sampling_config))
        if not out.output_text:
            out.output_text = self.tok.decode(out.output_ids.tolist())
        env = MathEnv(self, conversation, str(conversation.extra.get("answer", "")), max_length=len(ids) + len(out.output_ids) + 1)
        _, _, _, trace, metric = await env.step(out)
        return RolloutResult(conversation=conversation, trace=trace, metric=metric)

    def build_sft_samples(self, dataset: Any) -> list:
        """Prompt + reference solution (``extra['solution']`` or the answer) as an SFT sample."""
        from axrl_b200.data.sample import Sample

        out = []
        for c in dataset.conversations:
            target = str(c.extra.get("solution") or c.extra.get("answer", ""))
            resp = self.tok.tok.encode(target) if hasattr(self.tok.tok, "encode") else []
            out.append(Sample.from_tokens([int(t) for t in c.gen_state.input_ids], list(resp) + [int(self.tok.eos_id)]))
        return out


class Gsm8kRecipe(SingleTurnQARecipe):
    def __init__(self, config: Any, tokenizer: Any, train_path: str | None = None, test_path: str | None = None,
                 train: BaseDataset | None = None, test: BaseDataset | None = None) -> None:
        train = train or ParquetQADataset(train_path, question_key="question", answer_key="answer")
        test = test or (ParquetQADataset(test_path, question_key="question", answer_key="answer") if test_path else None)
        super().__init__(config, tokenizer, train, test)

    def score(self, text: str, answer: str) -> float:
        gt = answer.split("####")[-1].strip().replace(",", "")
        return compute_score(text, gt, method="flexible")
