"""Supervised fine-tuning loss (reference ``axrl/trainer/sft_trainer.py:20-100``): token-mean NLL on loss tokens."""

from __future__ import annotations

from axrl_b200.configs import SftTrainerConfig
from axrl_b200.trainer.base_trainer import BaseTrainer, aggregate_with_mask, denominator_count


class SftTrainer(BaseTrainer):
    def __init__(self, config: SftTrainerConfig) -> None:
        self.config = config

    def loss_func(self, outputs: dict, batch, with_metrics: bool = True):  # noqa: ANN001, ANN201
        m = batch["loss_mask"]
        metrics: dict[str, float] = {}
        if self.config.compute_entropy and "entropy" in outputs:
            metrics["entropy"] = float(aggregate_with_mask(outputs["entropy"], m, "token-mean"))
        if self.config.compute_accuracy and "argmax" in outputs:
            metrics["accuracy"] = float(aggregate_with_mask((outputs["argmax"] == batch["labels"]).float(), m, "token-mean"))
        loss = aggregate_with_mask(-outputs["log_prob"], m, "token-mean")
        denom = denominator_count(m, "token-mean")
        if with_metrics:
            metrics["denom"] = float(denom)
            metrics["loss"] = float(loss.detach())
        return loss, denom, metrics

    def compute_micro_batch_denominator(self, mask, num_turns: int = 0):  # noqa: ANN001, ANN201
        return denominator_count(mask, "token-mean")
