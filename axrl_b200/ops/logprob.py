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


def logprob_ref(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0, compute_entropy: bool = False,
                entropy_top_k: int = 0):  # noqa: ANN201
    logits = torch.nn.functional.linear(hidden.float(), weight.float()) / temperature
    lse = torch.logsumexp(logits, -1)
    lab = labels.long().clamp(min=0)
    lp = logits.gather(-1, lab[:, None]).squeeze(-1) - lse
    ent = None
    if compute_entropy:
        el = logits
        if entropy_top_k > 0:  # entropy of the top-k masked distribution
            kth = torch.topk(logits, entropy_top_k, -1).values[:, -1:]
            el = logits.masked_fill(logits < kth, float("-inf"))
        p = torch.softmax(el, -1)
        ent = torch.logsumexp(el, -1) - (p * el.nan_to_num(neginf=0.0)).sum(-1)
    return lp, ent


@torch.no_grad()
def argmax_tokens(hidden: torch.Tensor, weight: torch.Tensor, chunk: int = DEFAULT_CHUNK) -> torch.Tensor:
    """Most likely next token per row (SFT accuracy), chunked like the log-prob op."""
    out = torch.empty(hidden.shape[0], dtype=torch.int64, device=hidden.device)
    for s in range(0, hidden.shape[0], chunk):
        h = hidden[s:s + chunk]
        logits = _ext.ext().linear_fwd(h.contiguous(), weight) if h.is_cuda else torch.nn.functional.linear(h, weight)
        out[s:s + chunk] = logits.argmax(-1)
    return out


class _FusedLogprob(torch.autograd.Function):
    """``topk > 0``: the entropy is that of the softmax restricted to each row's ``topk`` largest
    (temperature-scaled) logits — the reference's top-k masked entropy — and its gradient is
    scattered onto those columns of the chunk's dlogits."""

    @staticmethod
    def forward(ctx, hidden, weight, labels, temperature, compute_entropy, chunk, topk=0):  # noqa: ANN001, ANN205
        e = _ext.ext()
        T = hidden.shape[0]
        lp = torch.empty(T, dtype=torch.float32, device=hidden.device)
        lse = torch.empty(T, dtype=torch.float32, device=hidden.device)
        full_ent = compute_entropy and topk <= 0
        ent = torch.empty(T if compute_entropy else 0, dtype=torch.float32, device=hidden.device)
        idx = torch.empty((T, topk) if (compute_entropy and topk > 0) else (0, 0), dtype=torch.int64, device=hidden.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            e.logprob_fwd(logits, labels[s:s + t], temperature, lp[s:s + t], lse[s:s + t], ent[s:s + t] if full_ent else ent[:0])
            if compute_entropy and topk > 0:
                vals, ix = torch.topk(logits, topk, dim=-1)
                z = vals.float() / temperature
                pk = torch.softmax(z, -1)
                ent[s:s + t] = torch.logsumexp(z, -1) - (pk * z).sum(-1)
                idx[s:s + t] = ix
        ctx.save_for_backward(hidden, weight, labels, lse, ent, idx)
        ctx.cfg = (temperature, compute_entropy, chunk, topk)
        return lp, (ent if compute_entropy else None)

    @staticmethod
    def backward(ctx, g_lp, g_ent):  # noqa: ANN001, ANN205
        hidden, weight, labels, lse, ent, idx = ctx.saved_tensors
        temperature, compute_entropy, chunk, topk = ctx.cfg
        e = _ext.ext()
        T = hidden.shape[0]
        g_lp = torch.zeros(T, dtype=torch.float32, device=hidden.device) if g_lp is None else g_lp.float().contiguous()
        use_ent = compute_entropy and g_ent is not None and topk <= 0
        use_topk = compute_entropy and g_ent is not None and topk > 0
        g_ent_t = g_ent.float().contiguous() if (use_ent or use_topk) else torch.empty(0, device=hidden.device)
        dh = torch.empty_like(hidden)
        main = getattr(weight, "main_grad", None)
        dw = None if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        for s in range(0, T, chunk):
            t = min(chunk, T - s)
            logits = e.linear_fwd(hidden[s:s + t], weight)
            if use_topk:  # d H_k / d z_j = -p_j (z_j - E_k[z]) on the row's top-k columns
                ix = idx[s:s + t]
                z = logits.gather(1, ix).float() / temperature
                pk = torch.softmax(z, -1)
                dz = -pk * (z - (pk * z).sum(-1, keepdim=True)) * g_ent_t[s:s + t, None] / temperature
            empty = torch.empty(0, device=hidden.device)
            e.logprob_bwd(logits, labels[s:s + t], lse[s:s + t], g_lp[s:s + t],
                          ent[s:s + t] if use_ent else empty, g_ent_t[s:s + t] if use_ent else empty, temperature)
            if use_topk:
                logits.scatter_add_(1, ix, dz.to(logits.dtype))
            dh[s:s + t] = e.linear_dgrad(logits, weight)
            e.linear_wgrad_acc(logits, hidden[s:s + t], main if main is not None else dw)
        return dh, (None if dw is None else dw.to(weight.dtype)), None, None, None, None, None


def fused_logprob(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0,
                  compute_entropy: bool = False, chunk: int = DEFAULT_CHUNK, entropy_top_k: int = 0):  # noqa: ANN201
    """Per-token ``log p(label)`` (fp32) and optional entropy (of the top-k masked distribution when
    ``entropy_top_k > 0``) from final hidden states."""
    if not hidden.is_cuda:
        return logprob_ref(hidden, weight, labels, temperature, compute_entropy, entropy_top_k)
    return _FusedLogprob.apply(hidden.contiguous(), weight, labels.to(torch.int32).contiguous(), float(temperature), bool(compute_entropy),
                               int(chunk), int(max(0, entropy_top_k)))


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
