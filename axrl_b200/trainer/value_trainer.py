"""PPO critic trainer (reference ``axrl/trainer/value_trainer.py:23-141``): clipped value loss on loss tokens."""

from __future__ import annotations

import torch
from torch import nn

from axrl_b200.configs import PPOValueConfig
from axrl_b200.trainer.base_trainer import BaseTrainer, aggregate_with_mask, denominator_count
from axrl_b200.trainer.ppo_utils import clipped_value_loss_per_token


class ValueHead(nn.Module):
    """Linear hidden -> scalar value (reference ``axrl/utils/megatron/value_head.py:16-63``)."""

    def __init__(self, hidden: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(1, hidden))

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.linear(h.float(), self.weight.float()).squeeze(-1)


class ValueTrainer(BaseTrainer):
    def __init__(self, config: PPOValueConfig) -> None:
        self.config = config

    def compute_micro_batch_denominator(self, mask, num_turns: int = 0):  # noqa: ANN001, ANN201
        """The value loss is a token mean over loss tokens."""
        return denominator_count(mask, "token-mean")

    def loss_func(self, outputs: dict, batch, with_metrics: bool = True):  # noqa: ANN001, ANN201
        values = outputs["values"]
        m = batch["loss_mask"].bool()
        losses, clipfrac = clipped_value_loss_per_token(values, batch["old_values"], batch["returns"], value_clip=self.config.value_clip)
        loss = aggregate_with_mask(losses, m, "token-mean") * self.config.value_loss_coef
        denom = denominator_count(m, "token-mean")
        metrics: dict[str, float] = {}
        if with_metrics:
            def agg(v, mode):  # noqa: ANN001, ANN202
                return float(aggregate_with_mask(v.float(), m, mode)) if m.any() else 0.0

            lv = float(loss.detach())
            metrics = {"loss": lv, "value_loss": lv, "denom": float(denom), "num_samples": float(values.shape[0]),
                       "value_mean": agg(values, "token-mean"), "value_std": agg(values, "token-std"),
                       "return_mean": agg(batch["returns"], "token-mean"), "return_std": agg(batch["returns"], "token-std")}
            if clipfrac is not None:
                metrics["value_clipfrac"] = agg(clipfrac, "token-mean")
        return loss, denom, metrics
