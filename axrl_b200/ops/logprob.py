"""Fused LM-head log-probability (+ entropy) without materialising full logits.

Replaces the reference's ``logits.float()`` -> ``vocab_parallel_log_prob`` /
``vocab_parallel_entropy`` chain (``axrl/utils/megatron/tensor_parallel.py:8-82``,
``axrl/trainer/grpo_trainer.py:805-825``), which holds a (T, V) fp32 tensor.

Tokens are processed in chunks of ``chunk`` rows: one GEMM produces bf16
logits for the chunk, then one kernel per row computes (in fp32, with the
temperature applied) the log-sum-exp, the label log-prob and optionally the
entropy.  Backward recomputes each chunk's logits and turns them in place into
``dlogits = (onehot - softmax) * g_lp / t  - softmax * (s - E[s]) * g_ent / t``
before the two gradient GEMMs.  Peak extra memory is one (chunk, V) bf16 tile.

With tensor parallelism over the vocabulary the per-row (max, sum-exp,
label-logit) triples are combined across ranks (see
:mod:`axrl_b200.parallel.vocab`).
"""

from __future__ import annotations

import torch

from axrl_b200.ops import _ext

DEFAULT_CHUNK = 4096


def logprob_ref(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0, compute_entropy: bool = False):  # noqa: ANN201
    logits = torch.nn.functional.linear(hidden.float(), weight.float()) / temperature
    lse = torch.logsumexp(logits, -1)
    lab = labels.long().clamp(min=0)
    lp = logits.gather(-1, lab[:, None]).squeeze(-1) - lse
    ent = None
    if compute_entropy:
        p = torch.softmax(logits, -1)
        ent = lse - (p * logits).sum(-1)
    return lp, ent


class _FusedLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, temperature, compute_entropy, chunk):  # noqa: ANN001, ANN205
        e = _ext.ext()
        T = hidden.shape[0]
        lp = torch.empty(T, dtype=torch.float32, device=hidden.device)
        lse = torch.empty(T, dtype=torch.float32, device=hidden.device)
        ent = torch.empty(T if compute_entropy else 0, dtype=torch.float32, device=hidden.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            e.logprob_fwd(logits, labels[s:s + t], temperature, lp[s:s + t], lse[s:s + t], ent[s:s + t] if compute_entropy else ent)
        ctx.save_for_backward(hidden, weight, labels, lse, ent)
        ctx.cfg = (temperature, compute_entropy, chunk)
        return lp, (ent if compute_entropy else None)

    @staticmethod
    def backward(ctx, g_lp, g_ent):  # noqa: ANN001, ANN205
        hidden, weight, labels, lse, ent = ctx.saved_tensors
        temperature, compute_entropy, chunk = ctx.cfg
        e = _ext.ext()
        T = hidden.shape[0]
        g_lp = torch.zeros(T, dtype=torch.float32, device=hidden.device) if g_lp is None else g_lp.float().contiguous()
        use_ent = compute_entropy and g_ent is not None
        g_ent_t = g_ent.float().contiguous() if use_ent else torch.empty(0, device=hidden.device)
        dh = torch.empty_like(hidden)
        main = getattr(weight, "main_grad", None)
        dw = None if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            e.logprob_bwd(logits, labels[s:s + t], lse[s:s + t], g_lp[s:s + t],
                          ent[s:s + t] if use_ent else ent, g_ent_t[s:s + t] if use_ent else g_ent_t, temperature)
            dh[s:s + t] = e.linear_dgrad(logits, weight)
            e.linear_wgrad_acc(logits, hidden[s:s + t], main if main is not None else dw)
        return dh, (None if dw is None else dw.to(weight.dtype)), None, None, None, None


def fused_logprob(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0,
                  compute_entropy: bool = False, chunk: int = DEFAULT_CHUNK):  # noqa: ANN201
    """Per-token ``log p(label)`` (fp32) and optional entropy from final hidden states."""
    if not hidden.is_cuda:
        return logprob_ref(hidden, weight, labels, temperature, compute_entropy)
    return _FusedLogprob.apply(hidden.contiguous(), weight, labels.to(torch.int32).contiguous(), float(temperature), bool(compute_entropy), int(chunk))


class _FusedLogprobVP(torch.autograd.Function):
    """Vocabulary-parallel variant: ``weight`` holds rows [v0, v0 + Vs) of the LM head.  Per chunk
    the local kernel yields (lse_r, label logit or 0, E_r[s]); the per-token triples of all TP ranks
    are combined once for the whole micro-batch.  Backward runs the local kernel with the GLOBAL
    lse / entropy, giving this rank's slice of dlogits; ``dh`` is a partial sum over ranks."""

    @staticmethod
    def forward(ctx, hidden, weight, labels_local, inside, temperature, compute_entropy, chunk, comm):  # noqa: ANN001, ANN205
        from axrl_b200.parallel.tensor_parallel import combine_vocab_stats

        e = _ext.ext()
        T = hidden.shape[0]
        lp_r = torch.empty(T, dtype=torch.float32, device=hidden.device)
        lse_r = torch.empty(T, dtype=torch.float32, device=hidden.device)
        ent_r = torch.empty(T, dtype=torch.float32, device=hidden.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            e.logprob_fwd(logits, labels_local[s:s + t], temperature, lp_r[s:s + t], lse_r[s:s + t], ent_r[s:s + t])
        lab_r = torch.where(inside, lp_r + lse_r, torch.zeros_like(lp_r))
        es_r = lse_r - ent_r if compute_entropy else None
        lp, lse, ent = combine_vocab_stats(lse_r, lab_r, es_r, comm)
        ent_save = ent if ent is not None else torch.empty(0, device=hidden.device)
        ctx.save_for_backward(hidden, weight, labels_local, lse, ent_save)
        ctx.cfg = (temperature, compute_entropy, chunk)
        return lp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):  # noqa: ANN001, ANN205
        hidden, weight, labels, lse, ent = ctx.saved_tensors
        temperature, compute_entropy, chunk = ctx.cfg
        e = _ext.ext()
        T = hidden.shape[0]
        g_lp = torch.zeros(T, dtype=torch.float32, device=hidden.device) if g_lp is None else g_lp.float().contiguous()
        use_ent = compute_entropy and g_ent is not None
        g_ent_t = g_ent.float().contiguous() if use_ent else torch.empty(0, device=hidden.device)
        dh = torch.empty_like(hidden)
        main = getattr(weight, "main_grad", None)
        dw = None if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            e.logprob_bwd(logits, labels[s:s + t], lse[s:s + t], g_lp[s:s + t],
                          ent[s:s + t] if use_ent else ent, g_ent_t[s:s + t] if use_ent else g_ent_t, temperature)
            dh[s:s + t] = e.linear_dgrad(logits, weight)
            e.linear_wgrad_acc(logits, hidden[s:s + t], main if main is not None else dw)
        return dh, (None if dw is None else dw.to(weight.dtype)), None, None, None, None, None, None


def fused_logprob_vocab_parallel(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, v0: int, comm,  # noqa: ANN001
                                 temperature: float = 1.0, compute_entropy: bool = False, chunk: int = DEFAULT_CHUNK):  # noqa: ANN201
    Vs = weight.shape[0]
    lab = labels.long()
    loc = lab - v0
    inside = (loc >= 0) & (loc < Vs) & (lab >= 0)
    # local label: index in the shard; Vs (never a column) for trained rows owned elsewhere; -1 ignored
    local = torch.where(inside, loc, torch.where(lab >= 0, torch.full_like(loc, Vs), torch.full_like(loc, -1))).to(torch.int32)
    return _FusedLogprobVP.apply(hidden.contiguous(), weight, local.contiguous(), inside, float(temperature), bool(compute_entropy),
                                 int(chunk), comm)
