"""GRPO-family objectives: hand-computed golden values and gradient behaviour."""

import math

import pytest
import torch

from axrl_b200.configs import GrpoTrainerConfig
from axrl_b200.trainer.base_trainer import aggregate_with_mask
from axrl_b200.trainer.grpo_trainer import GrpoTrainer


def _batch(lp_old=0.0, adv=(1.0, -1.0), mask=(True, True), rollout=None):
    n = len(adv)
    b = {
        "loss_mask": torch.tensor([list(mask)]),
        "labels": torch.zeros(1, n, dtype=torch.long),
        "advantage": torch.tensor([list(adv)]),
        "old_logprobs": torch.full((1, n), lp_old),
        "ref_logprobs": torch.full((1, n), lp_old),
        "rollout_logprobs": torch.full((1, n), lp_old) if rollout is None else torch.tensor([list(rollout)]),
    }
    return b


def test_ppo_clip_golden():
    t = GrpoTrainer(GrpoTrainerConfig(loss_type="ppo", clip_ratio_high=0.2, clip_ratio_low=0.2, dual_clip_neg_adv_factor=None))
    lp = torch.log(torch.tensor([[1.5, 0.5]]))
    loss, denom, m = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, _batch())
    # token 0: adv 1, ratio 1.5 -> min(1.5, 1.2) objective -> loss -1.2 ; token 1: adv -1, ratio .5 -> max(-.5,-.8)... loss 0.8
    assert loss.item() == pytest.approx((-1.2 + 0.8) / 2)
    assert int(denom) == 2
    assert m["clip_frac__all"] == pytest.approx(1.0)
    assert m["ppo_policy_loss"] == pytest.approx(-0.2)


def test_ppo_requires_old_base():
    with pytest.raises(AssertionError, match="old_logprobs"):
        GrpoTrainer(GrpoTrainerConfig(loss_type="ppo", is_base_logprobs="rollout_logprobs")).get_loss_func()


def test_dual_clip_caps_negative_advantage():
    t = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo", clip_ratio_high=0.2, clip_ratio_low=0.2, dual_clip_neg_adv_factor=3.0))
    lp = torch.log(torch.tensor([[10.0]]))
    loss, _, _ = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, _batch(adv=(-1.0,), mask=(True,)))
    assert loss.item() == pytest.approx(3.0)  # min(3*1, 10*1)


def test_tis_and_kimi_gradients():
    for lt, base in (("tis", "old_logprobs"), ("kimi2_5", "rollout_logprobs")):
        t = GrpoTrainer(GrpoTrainerConfig(loss_type=lt, is_base_logprobs=base, clip_ratio_high=0.2, clip_ratio_low=0.2))
        lp = torch.log(torch.tensor([[2.0, 1.0]])).requires_grad_(True)
        loss, _, _ = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, _batch(adv=(1.0, 1.0)))
        loss.backward()
        g = lp.grad[0]
        # weight = clip(ratio, .8, 1.2) detached: token0 clipped to 1.2, token1 1.0 ; d(-adv*w*lp)/dlp = -w/2
        if lt == "tis":
            assert g[0].item() == pytest.approx(-0.6)
        else:  # hard clip stops gradient of clipped tokens
            assert g[0].item() == pytest.approx(0.0)
        assert g[1].item() == pytest.approx(-0.5)


def test_grpo2_quadrants():
    c = GrpoTrainerConfig(loss_type="grpo2", clip_ratio_high=0.28, clip_ratio_low=0.2, dual_soft_clip=3.0)
    t = GrpoTrainer(c)
    ratios = torch.tensor([[2.0, 0.5, 5.0, 0.5]])
    adv = (1.0, 1.0, -1.0, -1.0)
    lp = torch.log(ratios).requires_grad_(True)
    loss, _, _ = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, _batch(adv=adv, mask=(True,) * 4))
    loss.backward()
    g = lp.grad[0] * 4
    assert g[0].item() == pytest.approx(0.0)  # adv>=0, r>1: hard clip at 1.28 (clipped -> no grad)
    assert g[1].item() == pytest.approx(-0.5)  # adv>=0, r<=1: soft, w = r
    assert g[2].item() == pytest.approx(3.0)  # adv<0, r>1: soft clip at 3
    assert g[3].item() == pytest.approx(0.0)  # adv<0, r<=1: hard clip at 0.8 (clipped)


def test_gspo_sequence_ratio():
    t = GrpoTrainer(GrpoTrainerConfig(loss_type="gspo", loss_agg_type="seq-mean-token-mean", clip_ratio_high=10, clip_ratio_low=0.9))
    lp = torch.tensor([[math.log(2.0), 0.0]]).requires_grad_(True)
    loss, _, _ = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, _batch(adv=(1.0, 1.0)))
    assert loss.item() == pytest.approx(-math.sqrt(2.0), rel=1e-5)


def test_tis_weight_and_icepop_and_seq_mask():
    c = GrpoTrainerConfig(loss_type="grpo", mismatch_token_clip_max=2.0, icepop_masking_low=0.5, icepop_masking_high=5.0,
                          dual_clip_neg_adv_factor=None)
    t = GrpoTrainer(c)
    lp = torch.zeros(1, 3)
    b = _batch(adv=(1.0, 1.0, 1.0), mask=(True,) * 3)
    b["rollout_logprobs"] = torch.log(torch.tensor([[1 / 3.0, 1.0, 10.0]]))  # old/rollout ratio = 3, 1, 0.1
    loss, _, m = t.loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, b)
    # token0: ratio 3 -> tis clipped to 2, icepop keeps (3<5); token1 weight 1; token2: ratio .1 < .5 -> dropped
    assert loss.item() == pytest.approx(-(2.0 + 1.0) / 3)
    assert m["icepop_mask_low_ratio__all"] == pytest.approx(1 / 3)
    c2 = GrpoTrainerConfig(loss_type="grpo", mismatch_seq_masking_low=0.9, mismatch_seq_masking_high=1.1, dual_clip_neg_adv_factor=None)
    loss2, _, m2 = GrpoTrainer(c2).loss_func({"log_prob": lp, "entropy": torch.zeros_like(lp)}, b)
    assert loss2.item() == pytest.approx(0.0)  # geometric mean ratio far from 1 -> whole sequence masked
    assert m2["seq_mask_keep_rate__all"] == pytest.approx(0.0)


def test_aggregations():
    v = torch.tensor([[1.0, 2.0, 3.0], [4.0, 0.0, 0.0]])
    m = torch.tensor([[True, True, True], [True, False, False]])
    assert aggregate_with_mask(v, m, "token-mean").item() == pytest.approx(2.5)
    assert aggregate_with_mask(v, m, "seq-mean-token-mean").item() == pytest.approx(3.0)
    assert aggregate_with_mask(v, m, "token-max").item() == 4.0
    assert aggregate_with_mask(v, m, "token-min").item() == 1.0


def test_denominators_and_opd():
    from axrl_b200.configs import ModelConfig, OPDConfig

    c = GrpoTrainerConfig(micro_batch_denominator_type="sequence")
    t = GrpoTrainer(c)
    assert int(t.compute_micro_batch_denominator(torch.tensor([[True, False], [False, False]]))) == 1
    opd = OPDConfig(enabled=True, backend="megatron", teacher_model=ModelConfig(name="x"), opd_alpha=0.5, reverse_kl_clip=1.0)
    t2 = GrpoTrainer(GrpoTrainerConfig(opd=opd))
    adv = torch.tensor([[1.0, 1.0]])
    mask = torch.tensor([[True, True]])
    cur = torch.tensor([[-1.0, -1.0]])
    teacher = torch.tensor([[-1.5, -4.0]])
    new, m = t2.apply_opd_to_advantages(advantages=adv, loss_mask=mask, cur_logprobs=cur, rollout_logprobs=cur, old_logprobs=cur,
                                         teacher_logprobs=teacher)
    assert new[0, 0].item() == pytest.approx(0.5 * 1 - 0.5 * 0.5)
    assert new[0, 1].item() == pytest.approx(0.5 * 1 - 0.5 * 1.0)  # reverse KL 3 clipped to 1
    assert m["opd/reverse_kl_clip_rate"] == pytest.approx(0.5)


def test_topk_entropy_ref_and_sft_accuracy():
    from axrl_b200.ops.logprob import logprob_ref

    torch.manual_seed(0)
    h = torch.randn(5, 16)
    w = torch.randn(40, 16)
    lab = torch.randint(0, 40, (5,))
    _, e_full = logprob_ref(h, w, lab, compute_entropy=True)
    _, e_k = logprob_ref(h, w, lab, compute_entropy=True, entropy_top_k=4)
    logits = h @ w.t()
    top = torch.topk(logits, 4, -1).values
    p = torch.softmax(top, -1)
    torch.testing.assert_close(e_k, torch.logsumexp(top, -1) - (p * top).sum(-1))
    assert (e_k <= e_full + 1e-6).all() and (e_k <= torch.log(torch.tensor(4.0)) + 1e-6).all()
