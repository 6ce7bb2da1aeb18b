"""PPO helpers: terminal token rewards, reverse-scan GAE, batch normalisation, clipped value loss.

Reference: ``axrl/trainer/ppo_utils.py:6-107``.  GAE here is vectorised over the batch
and scans time once in reverse.
"""

from __future__ import annotations

import torch


def build_terminal_token_rewards(scores: torch.Tensor, loss_mask: torch.Tensor) -> torch.Tensor:
    """Scalar score on each row's last valid (loss) token, zeros elsewhere."""
    m = loss_mask.bool().to(scores.device)
    out = torch.zeros(m.shape, dtype=torch.float32, device=scores.device)
    has = m.any(1)
    if has.any():
        pos = torch.arange(m.shape[1], device=m.device).expand_as(m).masked_fill(~m, -1)
        last = pos.max(1).values
        rows = torch.nonzero(has).squeeze(1)
        out[rows, last[rows]] = scores.float()[rows]
    return out


@torch.no_grad()
def compute_gae(rewards: torch.Tensor, values: torch.Tensor, loss_mask: torch.Tensor, *, gamma: float = 1.0, gae_lambda: float = 1.0):  # noqa: ANN201
    """Token-level GAE restricted to valid tokens; a value bootstraps only from a valid next token."""
    assert rewards.shape == values.shape == loss_mask.shape
    r, v, m = rewards.float(), values.float(), loss_mask.bool()
    B, T = r.shape
    adv = torch.zeros_like(r)
    carry = torch.zeros(B, dtype=r.dtype, device=r.device)
    mf = m.float()
    for t in range(T - 1, -1, -1):
        nv = v[:, t + 1] if t + 1 < T else torch.zeros_like(carry)
        nm = mf[:, t + 1] if t + 1 < T else torch.zeros_like(carry)
        delta = r[:, t] + gamma * nv * nm - v[:, t]
        carry = (delta + gamma * gae_lambda * carry * nm) * mf[:, t]
        adv[:, t] = carry
    return adv.masked_fill(~m, 0.0), (adv + v).masked_fill(~m, 0.0)


def normalize_over_valid_tokens_in_batch(values: torch.Tensor, loss_mask: torch.Tensor, *, eps: float = 1e-8) -> torch.Tensor:
    m = loss_mask.bool()
    if not m.any():
        return torch.zeros_like(values)
    sel = values.float().masked_select(m)
    out = (values.float() - sel.mean()) * torch.rsqrt(sel.var(unbiased=False) + eps)
    return out.masked_fill(~m, 0.0)


def clipped_value_loss_per_token(values: torch.Tensor, old_values: torch.Tensor, returns: torch.Tensor, *, value_clip: float | None = 0.2):  # noqa: ANN201
    """max((v - R)^2, (clip(v, v_old +- c) - R)^2) and the fraction of tokens whose value moved more than c."""
    assert values.shape == old_values.shape == returns.shape
    v, vo, R = values.float(), old_values.float(), returns.float()
    unclipped = (v - R).pow(2)
    if value_clip is None:
        return unclipped, None
    clipped = (vo + (v - vo).clamp(-value_clip, value_clip) - R).pow(2)
    return torch.maximum(unclipped, clipped), ((v - vo).abs() > value_clip).float()
