"""DAPO17k math recipe (used with the Qwen3-30B-A3B MoE model and routing replay).

Reference: the DAPO17k MoE recipe of ``axis_recipe`` with the DAPO / Minerva reward
(``axrl/verifier/dapo_utils.py``).  Prompts come from a parquet file with ``prompt`` / ``answer``
columns; the reward is the strict boxed check (or Minerva ``Answer:`` matching).
"""

from __future__ import annotations

from typing import Any

from axrl_b200.datasets.base_dataset import BaseDataset, ParquetQADataset
from axrl_b200.recipe.gsm8k_recipe import SingleTurnQARecipe
from axrl_b200.verifier.dapo import compute_score

DAPO_PROMPT = ("Solve the following math problem step by step. The last line of your response should be of the form "
               "Answer: $Answer (without quotes) where $Answer is the answer to the problem.")


class DapoRecipe(SingleTurnQARecipe):
    def __init__(self, config: Any, tokenizer: Any, train_path: str | None = None, test_path: str | None = None,
                 train: BaseDataset | None = None, test: BaseDataset | None = None, strict_box_verify: bool = False) -> None:
        train = train or ParquetQADataset(train_path, question_key="prompt", answer_key="answer")
        test = test or (ParquetQADataset(test_path, question_key="prompt", answer_key="answer") if test_path else None)
        self.strict = strict_box_verify
        super().__init__(config, tokenizer, train, test, system_prompt=DAPO_PROMPT)

    def score(self, text: str, answer: str) -> float:
        return compute_score(text, answer, strict_box_verify=self.strict)
