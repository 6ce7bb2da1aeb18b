"""GRPO-family policy objectives.

Semantics follow reference ``axrl/trainer/grpo_trainer.py:50-803``:

* loss types ``grpo``/``ppo`` (PPO clip + optional dual clip on negative
  advantages), ``grpo2`` (four ratio/advantage quadrants, hard clip where the
  update moves away from the behaviour policy, soft clip where it moves back),
  ``tis`` / ``kimi2_5`` (REINFORCE weighted by a truncated, detached IS ratio;
  kimi2_5 stops the gradient of clipped tokens), ``topr`` and ``gspo``
  (sequence-level ratio);
* off-policy corrections computed from ``old - rollout`` logprobs: truncated
  token IS weight (TIS), geometric sequence mask with a min-token veto, IcePop
  token mask; they gate only the policy-gradient term;
* optional entropy control, k2 KL penalty and OPD advantage shaping;
* the micro-batch denominator (token / sequence / seq_turn) is returned with
  the loss so a caller can sum-then-divide across micro-batches and DP ranks.

Everything here works on padded ``(B, T)`` tensors and is the numerical
oracle.  The GPU training path evaluates the same objective on packed tokens
with the fused kernel in ``axrl_b200.ops.grpo_loss``; tests pin the two together.
"""

from __future__ import annotations

from typing import Callable

import torch

from axrl_b200.configs import GrpoTrainerConfig, ValueAggType
from axrl_b200.trainer.base_trainer import BaseTrainer, aggregate_with_mask
from axrl_b200.utils import kl_utils

LOG_RATIO_CLAMP = 20.0


def get_num_turns(turn_index: torch.Tensor, mask: torch.Tensor) -> int:
    """Number of distinct non-negative turn ids under ``mask``, summed over rows."""
    total = 0
    for row, m in zip(turn_index, mask):
        ids = row[m.bool()]
        total += int(ids[ids >= 0].unique().numel())
    return total


def _ratio(logprobs: torch.Tensor, base: torch.Tensor) -> torch.Tensor:
    return torch.exp((logprobs - base).clamp(-LOG_RATIO_CLAMP, LOG_RATIO_CLAMP))


def _implied_clip_ratio(pg_losses: torch.Tensor, adv: torch.Tensor) -> torch.Tensor:
    """Effective ratio implied by a per-token loss ``-adv * r`` (1 where adv ~ 0)."""
    return torch.where(adv.abs() < 1e-4, torch.ones_like(pg_losses), pg_losses / (-adv))


def _weighted_reinforce(
    ratio: torch.Tensor,
    logprobs: torch.Tensor,
    adv: torch.Tensor,
    mask: torch.Tensor,
    lo: float | None,
    hi: float | None,
    *,
    hard: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``-adv * clip(ratio) * logprob`` on ``mask``; ``hard`` detaches clipped tokens."""
    w = torch.clamp(ratio, min=0.0 if lo is None else lo, max=hi).detach()
    loss = -adv * w * logprobs
    if hard:
        loss = torch.where((ratio - w).abs() > 1e-5, loss.detach(), loss)
    zero = torch.zeros_like(loss)
    return torch.where(mask, loss, zero), torch.where(mask, w, torch.zeros_like(w))


class GrpoTrainer(BaseTrainer):
    def __init__(self, config: GrpoTrainerConfig) -> None:
        super().__init__()
        self.config = config

    # ------------------------------------------------------------------ denominators
    def compute_micro_batch_denominator(self, mask: torch.Tensor, num_turns: int = 0) -> torch.Tensor:
        kind = self.config.micro_batch_denominator_type
        if kind == "token":
            return mask.sum(dtype=torch.int)
        n_seq = (mask.sum(-1) > 0).sum(dtype=torch.int)
        if kind == "sequence":
            return n_seq
        if kind == "seq_turn":
            alpha = self.config.seq_turn_alpha if self.config.seq_turn_alpha is not None else self.config.turn_reward_alpha
            return (n_seq.float() + alpha * num_turns).to(torch.int)
        raise ValueError(kind)

    # ------------------------------------------------------------------ policy losses
    def grpo_loss(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        c = self.config
        if logprobs.is_cuda:  # fused kernel: ratio, clips, IS weight and gradient in one pass
            from axrl_b200.ops.grpo_loss import grpo_policy_loss

            if c.dual_clip_neg_adv_factor is not None:
                assert c.dual_clip_neg_adv_factor > 1.0
            pgw, ratio, eff = grpo_policy_loss(logprobs, base_logprobs, advantages, token_mismatch_tir, c.clip_ratio_low,
                                               c.clip_ratio_high, c.dual_clip_neg_adv_factor)
            return aggregate_with_mask(pgw, loss_mask, c.loss_agg_type), ratio, eff
        ratio = _ratio(logprobs, base_logprobs)
        clipped = torch.clamp(ratio, 1 - c.clip_ratio_low, 1 + c.clip_ratio_high)
        ppo = torch.maximum(-advantages * ratio, -advantages * clipped)
        if c.dual_clip_neg_adv_factor is None:
            pg = ppo
        else:
            assert c.dual_clip_neg_adv_factor > 1.0
            pg = torch.where(advantages < 0, torch.minimum(-c.dual_clip_neg_adv_factor * advantages, ppo), ppo)
        eff = _implied_clip_ratio(pg, advantages)
        return aggregate_with_mask(pg * token_mismatch_tir, loss_mask, c.loss_agg_type), ratio, eff

    def _reinforce_family(self, loss_mask, advantages, logprobs, base_logprobs, tir, *, hard: bool):  # noqa: ANN001
        c = self.config
        ratio = _ratio(logprobs, base_logprobs).detach()
        loss, w = _weighted_reinforce(ratio, logprobs, advantages, loss_mask, 1 - c.clip_ratio_low, 1 + c.clip_ratio_high, hard=hard)
        return aggregate_with_mask(loss * tir, loss_mask, c.loss_agg_type), ratio, w

    def tis_loss(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        return self._reinforce_family(loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir, hard=False)

    def kimi2_5_loss(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        return self._reinforce_family(loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir, hard=True)

    def topr_loss(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        ratio = _ratio(logprobs, base_logprobs).detach()
        pos = (advantages >= 0) & loss_mask
        neg = (advantages < 0) & loss_mask
        l1, w1 = _weighted_reinforce(ratio, logprobs, advantages, pos, 1.0, 1.0, hard=False)
        l2, w2 = _weighted_reinforce(ratio, logprobs, advantages, neg, 0.0, 1.0, hard=False)
        loss = (l1 + l2) * token_mismatch_tir
        return aggregate_with_mask(loss, loss_mask, self.config.loss_agg_type), ratio, w1 + w2

    def grpo2_loss(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        c = self.config
        assert c.dual_soft_clip is not None
        ratio = _ratio(logprobs, base_logprobs).detach()
        pos, up = advantages >= 0, ratio > 1
        quads = (
            # (mask, lo, hi, hard)
            (pos & up & loss_mask, None, 1 + c.clip_ratio_high, True),
            (pos & ~up & loss_mask, 0.0, None, False),
            (~pos & up & loss_mask, None, c.dual_soft_clip, False),
            (~pos & ~up & loss_mask, 1 - c.clip_ratio_low, None, True),
        )
        loss = torch.zeros_like(logprobs)
        w = torch.zeros_like(ratio)
        for m, lo, hi, hard in quads:
            li, wi = _weighted_reinforce(ratio, logprobs, advantages, m, lo, hi, hard=hard)
            loss, w = loss + li, w + wi
        return aggregate_with_mask(loss * token_mismatch_tir, loss_mask, c.loss_agg_type), ratio, w

    def gspo(self, *, loss_mask, advantages, logprobs, base_logprobs, token_mismatch_tir):  # noqa: ANN001
        c = self.config
        assert c.loss_agg_type == "seq-mean-token-mean", "GSPO requires seq-mean-token-mean aggregation."
        lens = loss_mask.sum(-1).clamp(min=1)
        seq_lr = ((logprobs - base_logprobs) * loss_mask).sum(-1) / lens
        log_r = (logprobs - logprobs.detach() + seq_lr.detach()[:, None]).clamp(max=10.0)
        r = torch.exp(log_r)
        pg = torch.maximum(-advantages * r, -advantages * r.clamp(1 - c.clip_ratio_low, 1 + c.clip_ratio_high))
        eff = _implied_clip_ratio(pg, advantages)
        return aggregate_with_mask(pg * token_mismatch_tir, loss_mask, c.loss_agg_type), r, eff

    def get_loss_func(self) -> Callable:
        lt = self.config.loss_type
        if lt == "ppo":
            assert self.config.is_base_logprobs == "old_logprobs", "PPO needs old_logprobs as ratio base."
        if lt == "kimi2_5":
            assert self.config.is_base_logprobs == "rollout_logprobs" and self.config.mismatch_token_clip_max is None
        table = {
            "grpo": self.grpo_loss, "ppo": self.grpo_loss, "tis": self.tis_loss, "grpo2": self.grpo2_loss,
            "topr": self.topr_loss, "gspo": self.gspo, "kimi2_5": self.kimi2_5_loss,
        }
        if lt not in table:
            raise ValueError(f"Unsupported loss type: {lt}")
        return table[lt]

    # ------------------------------------------------------------------ off-policy corrections
    def get_ratio(self, logprobs: torch.Tensor, base_logprobs: torch.Tensor) -> torch.Tensor:
        return _ratio(logprobs, base_logprobs)

    def get_seq_ratio(self, logprobs: torch.Tensor, base_logprobs: torch.Tensor, loss_mask: torch.Tensor) -> torch.Tensor:
        lr = ((logprobs - base_logprobs) * loss_mask).clamp(-LOG_RATIO_CLAMP, LOG_RATIO_CLAMP)
        seq = (lr.sum(-1) / loss_mask.sum(-1).clamp(min=1.0)).clamp(-LOG_RATIO_CLAMP, LOG_RATIO_CLAMP)
        return torch.exp(seq)[:, None].expand_as(lr)

    def truncate_mismatch_token_ratio(self, old_logprobs, rollout_logprobs, loss_mask, advantages):  # noqa: ANN001
        ir = _ratio(old_logprobs, rollout_logprobs).detach()
        ir = torch.where(loss_mask, ir, torch.ones_like(ir))
        cmax = self.config.mismatch_token_clip_max
        tir = torch.ones_like(ir) if cmax is None else ir.clamp(max=cmax)
        applied = torch.zeros_like(tir) if cmax is None else ((tir - ir).abs() > 1e-4).float()
        m: dict[str, float] = {}
        m.update(self.group_metrics(ir, "token_mismatch_ir", loss_mask, advantages))
        m.update(self.group_metrics(ir, "token_mismatch_ir_batch_max", loss_mask, advantages, mode="token-max"))
        m.update(self.group_metrics(ir, "token_mismatch_ir_batch_min", loss_mask, advantages, mode="token-min"))
        m.update(self.group_metrics(applied, "token_mismatch_ir_clip_rate", loss_mask, advantages))
        return ir, tir, m

    def get_icepop_token_mask(self, token_mismatch_ir, loss_mask, advantages):  # noqa: ANN001
        lo, hi = self.config.icepop_masking_low, self.config.icepop_masking_high
        low = token_mismatch_ir < lo if lo is not None else torch.zeros_like(loss_mask)
        high = token_mismatch_ir > hi if hi is not None else torch.zeros_like(loss_mask)
        drop = low | high
        m: dict[str, float] = {}
        for v, name in ((low, "icepop_mask_low_ratio"), (high, "icepop_mask_high_ratio"), (drop, "icepop_mask_ratio"), (~drop, "icepop_keep_ratio")):
            m.update(self.group_metrics(v.float(), name, loss_mask, advantages))
        return ~drop, m

    def get_mismatch_sequence_mask(self, token_mismatch_ir, logprobs, rollout_logprobs, loss_mask, advantages):  # noqa: ANN001
        c = self.config
        sr = self.get_seq_ratio(logprobs, rollout_logprobs, loss_mask).detach()
        ones = torch.ones_like(loss_mask)
        low = sr >= c.mismatch_seq_masking_low if c.mismatch_seq_masking_low is not None else ones
        high = sr <= c.mismatch_seq_masking_high if c.mismatch_seq_masking_high is not None else ones
        seq_min = token_mismatch_ir.min(-1, keepdim=True).values
        veto = (seq_min >= c.mismatch_token_veto_threshold) if c.mismatch_token_veto_threshold is not None else torch.ones_like(seq_min, dtype=torch.bool)
        veto = veto.expand_as(loss_mask)
        keep = low & high & veto
        m: dict[str, float] = {}
        for v, name in ((low, "seq_mask_low_keep_rate"), (high, "seq_mask_high_keep_rate"), (veto, "seq_mask_veto_keep_rate"), (keep, "seq_mask_keep_rate")):
            m.update(self.group_metrics(v.float(), name, loss_mask, advantages))
        m.update(self.group_metrics(sr, "seq_ratio_batch_max", loss_mask, advantages, mode="token-max"))
        m.update(self.group_metrics(sr, "seq_ratio_batch_min", loss_mask, advantages, mode="token-min"))
        m.update(self.group_metrics(sr, "seq_ratio", loss_mask, advantages))
        return keep, m

    # ------------------------------------------------------------------ entropy / KL / OPD
    def get_top_entropy_mask(self, loss_mask: torch.Tensor, entropy: torch.Tensor, top_quantile: float) -> torch.Tensor:
        assert 0.0 < top_quantile < 1.0
        vals = entropy.detach().clone()
        vals[~loss_mask] = torch.finfo(vals.dtype).min
        ks = torch.ceil(loss_mask.sum(1).float() * top_quantile).long().clamp(min=1)
        top, _ = torch.topk(vals, k=int(ks.max()), dim=1)
        thr = top[torch.arange(top.size(0)), ks - 1]
        return (vals >= thr[:, None]) & loss_mask

    def get_entropy_loss(self, entropy: torch.Tensor, loss_mask: torch.Tensor) -> tuple[torch.Tensor, float]:
        ec = self.config.entropy_control
        if ec.top_quantile < 1.0:
            loss_mask = self.get_top_entropy_mask(loss_mask, entropy, ec.top_quantile)
        ent = aggregate_with_mask(entropy, loss_mask, self.config.loss_agg_type)
        if ec.alpha <= 0.0:
            return torch.zeros((), device=entropy.device), float(ent)
        return (ec.target_entropy - ent) ** 2, float(ent)

    def get_kl_loss(self, logprobs: torch.Tensor, base_logprobs: torch.Tensor, loss_mask: torch.Tensor) -> torch.Tensor:
        return aggregate_with_mask(kl_utils.kl_divergence(logprobs, base_logprobs, "k2"), loss_mask, self.config.loss_agg_type)

    def apply_opd_to_advantages(self, *, advantages, loss_mask, cur_logprobs, rollout_logprobs, old_logprobs, teacher_logprobs):  # noqa: ANN001
        """Reverse-KL shaping: ``adv' = (1-a) adv - a * clip(student - teacher)`` on masked tokens."""
        oc = self.config.opd
        if not oc.enabled:
            return advantages, {}
        mask = loss_mask.bool()
        student = {"rollout_logprobs": rollout_logprobs, "old_logprobs": old_logprobs, "cur_logprobs": cur_logprobs}[oc.student_logprob_source]
        assert torch.isfinite(teacher_logprobs[mask]).all() and torch.isfinite(student[mask]).all()
        agg = aggregate_with_mask
        raw_s = agg(student.abs(), loss_mask, "token-mean")
        raw_t = agg(teacher_logprobs.abs(), loss_mask, "token-mean")
        scale = torch.ones((), device=student.device, dtype=student.dtype)
        if oc.normalize_student_logprob_scale:
            scale = raw_t / raw_s.clamp_min(1e-6)
            student = student * scale.detach()
        rkl = torch.where(mask, (student - teacher_logprobs).detach(), torch.zeros_like(advantages))
        raw_rkl = rkl
        if oc.reverse_kl_clip is not None:
            rkl = rkl.clamp(-oc.reverse_kl_clip, oc.reverse_kl_clip)
        adj = torch.where(mask, (1.0 - oc.opd_alpha) * advantages - oc.opd_alpha * rkl, advantages)
        ms = torch.where(mask, student, torch.zeros_like(student))
        mt = torch.where(mask, teacher_logprobs, torch.zeros_like(teacher_logprobs))
        metrics = {
            "opd/reverse_kl_mean": agg(rkl, loss_mask, "token-mean").item(),
            "opd/reverse_kl_std": agg(rkl, loss_mask, "token-std").item(),
            "opd/reverse_kl_abs_mean": agg(rkl.abs(), loss_mask, "token-mean").item(),
            "opd/reverse_kl_p05": agg(rkl, loss_mask, "token-p05").item(),
            "opd/reverse_kl_p95": agg(rkl, loss_mask, "token-p95").item(),
            "opd/reverse_kl_clip_rate": agg((rkl != raw_rkl).float(), loss_mask, "token-mean").item(),
            "opd/teacher_logprob_mean": agg(mt, loss_mask, "token-mean").item(),
            "opd/student_logprob_mean": agg(ms, loss_mask, "token-mean").item(),
            "opd/student_logprob_scale": float(scale),
            "opd/raw_student_teacher_logprob_abs_mean_ratio": (raw_s / raw_t.clamp_min(1e-6)).item(),
            "opd/student_teacher_logprob_abs_mean_ratio": (agg(ms.abs(), loss_mask, "token-mean") / agg(mt.abs(), loss_mask, "token-mean").clamp_min(1e-6)).item(),
            "opd/advantage_delta_mean": agg(adj - advantages, loss_mask, "token-mean").item(),
            "opd/base_advantage_mean": agg(advantages, loss_mask, "token-mean").item(),
            "opd/base_advantage_std": agg(advantages, loss_mask, "token-std").item(),
            "opd/adjusted_advantage_mean": agg(adj, loss_mask, "token-mean").item(),
            "opd/adjusted_advantage_std": agg(adj, loss_mask, "token-std").item(),
            "opd/teacher_logprobs_present_rate": agg(torch.where(mask, torch.isfinite(teacher_logprobs).float(), torch.zeros_like(advantages)), loss_mask, "token-mean").item(),
        }
        return adj, metrics

    # ------------------------------------------------------------------ metrics
    def group_metrics(self, values, prefix, mask, adv, mode: ValueAggType = "token-mean"):  # noqa: ANN001
        out = {f"{prefix}__all": aggregate_with_mask(values, mask, mode).item()}
        for tag, sel in (("pos", (adv > 0) & mask), ("neg", (adv < 0) & mask)):
            if sel.any():
                out[f"{prefix}__{tag}"] = aggregate_with_mask(values, sel, mode).item()
        return out

    def calculate_metrics(self, *, loss_mask, advantages, logprobs, rollout_logprobs, old_logprobs, ref_logprobs, entropy, ratio,
                          clipped_ratio, control_entropy, pg_loss, entropy_loss, kl_loss, loss):  # noqa: ANN001
        c = self.config
        agg = aggregate_with_mask
        m: dict[str, float] = {
            "pg_loss": pg_loss, "entropy_loss": entropy_loss, "kl_loss": kl_loss, "loss": loss,
            "control_entropy": control_entropy, "entropy_target": c.entropy_control.target_entropy,
            "entropy_alpha": c.entropy_control.alpha, "entropy_top_quantile": c.entropy_control.top_quantile,
            "kl_control_alpha": c.kl_control_alpha, "num_samples": advantages.shape[0],
            "perplexity": torch.exp(-agg(logprobs, loss_mask, "token-mean")).item(),
        }
        if c.loss_type == "ppo":
            m["ppo_policy_loss"] = pg_loss
        if not loss_mask.any():
            return m
        m.update(self.group_metrics((clipped_ratio - ratio).abs() > 1e-4, "clip_frac", loss_mask, advantages))
        m.update(self.group_metrics(ratio - clipped_ratio > 1e-4, "clip_frac_high", loss_mask, advantages))
        m.update(self.group_metrics(clipped_ratio - ratio > 1e-4, "clip_frac_low", loss_mask, advantages))

        def stats(v: torch.Tensor, name: str) -> None:
            for suf, mode in (("mean", "token-mean"), ("std", "token-std"), ("min", "token-min"), ("max", "token-max"), ("p05", "token-p05"), ("p95", "token-p95")):
                m[f"{name}_{suf}"] = agg(v, loss_mask, mode).item()

        probs = logprobs.exp()
        stats(entropy, "entropy")
        stats(ratio, "ratio")
        stats(probs, "prob")
        stats(_ratio(old_logprobs, rollout_logprobs), "ratio_mismatch")
        for lo10 in range(0, 18, 2):
            lo, hi = lo10 * 0.1, (lo10 + 2) * 0.1
            sel = (ratio >= lo) & (ratio < hi) & loss_mask
            if sel.any():
                m[f"prob_with_ratio_{lo:.1f}_{hi:.1f}"] = agg(probs, sel, "token-mean").item()
        sel = (ratio >= 2.0) & (ratio < 100.0) & loss_mask
        if sel.any():
            m["prob_with_ratio_2.0_100.0"] = agg(probs, sel, "token-mean").item()
        stats(kl_utils.kl_divergence(rollout_logprobs, old_logprobs, "k1"), "kl_k1_rollout_old")
        stats(kl_utils.kl_divergence(rollout_logprobs, old_logprobs, "k3"), "kl_k3_rollout_old")
        stats(kl_utils.kl_divergence(rollout_logprobs, old_logprobs, "k2"), "kl_k2_rollout_old")
        stats(kl_utils.kl_divergence(rollout_logprobs, logprobs, "k2"), "kl_k2_rollout_cur")
        stats(kl_utils.kl_divergence(old_logprobs, logprobs, "k2"), "kl_k2_old_cur")
        stats(kl_utils.kl_divergence(ref_logprobs, logprobs, "k2"), "kl_k2_ref_cur")
        m["intra_seq_ratio_std"] = agg(ratio, loss_mask, "seq-mean-token-std").item()
        return m

    # ------------------------------------------------------------------ loss closure
    def loss_func(self, outputs: dict[str, torch.Tensor], batch, with_metrics: bool = True):  # noqa: ANN001
        """Return ``(loss, denom, metrics)`` for one micro-batch of (B, T) tensors."""
        c = self.config
        loss_mask = batch["loss_mask"].bool()
        advantages = batch["advantage"]
        rollout_lp, old_lp = batch["rollout_logprobs"], batch["old_logprobs"]
        ref_lp = batch.get("ref_logprobs", None)
        if ref_lp is None:
            ref_lp = old_lp
        logprobs, entropy = outputs["log_prob"], outputs["entropy"]
        assert advantages.dim() == 2 and advantages.shape == logprobs.shape
        opd_metrics: dict[str, float] = {}
        if c.opd.enabled:
            teacher = batch.get("teacher_logprobs", None)
            assert teacher is not None, "OPD enabled but batch has no teacher_logprobs."
            advantages, opd_metrics = self.apply_opd_to_advantages(
                advantages=advantages, loss_mask=loss_mask, cur_logprobs=logprobs,
                rollout_logprobs=rollout_lp, old_logprobs=old_lp, teacher_logprobs=teacher)
        with torch.no_grad():
            ir, tir, m_tis = self.truncate_mismatch_token_ratio(old_lp, rollout_lp, loss_mask, advantages)
            ice_keep, m_ice = self.get_icepop_token_mask(ir, loss_mask, advantages)
            seq_keep, m_seq = self.get_mismatch_sequence_mask(ir, logprobs, rollout_lp, loss_mask, advantages)
        policy_tir = tir * seq_keep.to(tir.dtype) * ice_keep.to(tir.dtype)
        policy_mask = loss_mask & seq_keep & ice_keep
        base = old_lp if c.is_base_logprobs == "old_logprobs" else rollout_lp
        pg_loss, ratio, clipped = self.get_loss_func()(
            loss_mask=loss_mask, advantages=advantages, logprobs=logprobs, base_logprobs=base, token_mismatch_tir=policy_tir)
        ent_loss, ctrl_ent = self.get_entropy_loss(entropy, loss_mask)
        kl_base = old_lp if c.kl_base_logprobs == "old_logprobs" else ref_lp
        kl_loss = self.get_kl_loss(logprobs, kl_base, loss_mask)
        loss = pg_loss + ent_loss * c.entropy_control.alpha + kl_loss * c.kl_control_alpha
        turn_index = batch.get("turn_index", None)
        denom = self.compute_micro_batch_denominator(loss_mask, get_num_turns(turn_index, loss_mask) if turn_index is not None else 0)
        metrics: dict[str, float] = {}
        if with_metrics:
            with torch.no_grad():
                metrics = self.calculate_metrics(
                    loss_mask=policy_mask, advantages=advantages, logprobs=logprobs, rollout_logprobs=rollout_lp,
                    old_logprobs=old_lp, ref_logprobs=ref_lp, entropy=entropy, ratio=ratio, clipped_ratio=clipped,
                    control_entropy=ctrl_ent, pg_loss=pg_loss.item(), entropy_loss=float(ent_loss), kl_loss=kl_loss.item(), loss=loss.item())
                for d in (m_tis, m_ice, m_seq, opd_metrics):
                    metrics.update(d)
                metrics["loss_mask_sum"] = float(loss_mask.sum())
                metrics["policy_loss_mask_sum"] = float(policy_mask.sum())
                metrics["denom"] = float(denom)
        return loss, denom, metrics
