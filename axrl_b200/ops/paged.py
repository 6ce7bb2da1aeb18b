"""Inference-side ops over the paged KV cache (rollout engine).

Cache layout per layer: ``k_cache, v_cache: [num_pages, Hkv, page_size, D]``;
a token's slot is ``page * page_size + offset``.  CUDA tensors use the kernels
in ``csrc/kernels/decode_attn.cu`` / ``norm_act.cu`` / ``vocab.cu``; CPU
tensors use the PyTorch definitions here (oracle + CPU plumbing runs).
"""

from __future__ import annotations

import math
import os

import torch

from axrl_b200.ops import _ext
from axrl_b200.ops.core import _qk_norm_rope_ref, check_full_rotary

SPLIT_TOKENS = 128  # tokens per decode CTA (must match dec::SPLIT)


def _scatter_ref(cache: torch.Tensor, x: torch.Tensor, slots: torch.Tensor) -> None:
    P = cache.shape[2]
    page, off = slots // P, slots % P
    cache[page, :, off, :] = x.to(cache.dtype)


def qk_norm_rope_cache(qkv, qw, kw, pos, inv_freq, nq, nkv, eps, k_cache, v_cache, slots):  # noqa: ANN001, ANN201
    """q/k norm + RoPE and write k/v into the paged caches at ``slots``.  Returns q, k, v."""
    if not qkv.is_cuda:
        q, k, v = _qk_norm_rope_ref(qkv, qw, kw, pos, inv_freq, nq, nkv, eps)
        _scatter_ref(k_cache, k, slots.long())
        _scatter_ref(v_cache, v, slots.long())
        return q, k, v
    check_full_rotary(qw, inv_freq)
    return _ext.ext().qknorm_rope_cache(qkv, qw, kw, pos, inv_freq, nq, nkv, eps, k_cache, v_cache, slots)


def decode_attention_ref(q, k_cache, v_cache, block_table, seq_lens, scale):  # noqa: ANN001, ANN201
    B, Hq, D = q.shape
    Hkv, P = k_cache.shape[1], k_cache.shape[2]
    out = torch.zeros_like(q)
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            continue
        pages = block_table[b, : (n + P - 1) // P].long()
        k = k_cache[pages].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:n].float()
        v = v_cache[pages].permute(0, 2, 1, 3).reshape(-1, Hkv, D)[:n].float()
        rep = Hq // Hkv
        k = k.repeat_interleave(rep, 1)
        v = v.repeat_interleave(rep, 1)
        s = torch.einsum("hd,thd->ht", q[b].float(), k) * scale
        p = torch.softmax(s, -1)
        out[b] = torch.einsum("ht,thd->hd", p, v).to(q.dtype)
    return out


_FUSED_COMBINE = os.environ.get("AXRL_DECODE_FUSED_COMBINE", "0") == "1"


class DecodeWorkspace:
    """Split-KV partial buffers sized for (max_batch, Hq, max_context)."""

    def __init__(self, max_batch: int, hq: int, max_context: int, device) -> None:  # noqa: ANN001
        self.splits = max(1, math.ceil(max_context / SPLIT_TOKENS))
        self.part_o = torch.empty(max_batch * hq * self.splits * 128, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(max_batch * hq * self.splits * 2, dtype=torch.float32, device=device)
        # work lists of the planned decode kernels: 128-token splits, then 512-token chunks
        self.prefix = torch.zeros(2 * (max_batch + 1), dtype=torch.int32, device=device)
        # (sequence, kv head) chunk counters of the TMA decode kernel's fused combine (self-cleaning)
        self.chunk_cnt = torch.zeros(max_batch * hq, dtype=torch.int32, device=device)

    def plan(self, seq_lens: torch.Tensor) -> None:
        """Work list of live (sequence, split) pairs for ``seq_lens``; every layer of a step reuses it."""
        if seq_lens.is_cuda:
            _ext.ext().decode_plan(seq_lens, self.prefix)


def paged_decode_attention(q, k_cache, v_cache, block_table, seq_lens, ws: DecodeWorkspace | None, scale: float | None = None,  # noqa: ANN001, ANN201
                           planned: bool = False):
    """``planned=True``: ``ws.plan(seq_lens)`` already ran for these lengths (once per decode step)."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if not q.is_cuda:
        return decode_attention_ref(q, k_cache, v_cache, block_table, seq_lens, scale)
    out = torch.empty_like(q)
    if not planned:
        ws.plan(seq_lens)
    # the TMA kernel can merge its own chunks (AXRL_DECODE_FUSED_COMBINE=1), but the arrival handshake
    # per chunk cost more than the separate combine launch it saves (batch 64: 12.6 vs 8.8 ms per
    # Qwen3-8B decode step), so the combine kernel is the default
    _ext.ext().paged_decode_attn(q, k_cache, v_cache, block_table, seq_lens, out, ws.part_o, ws.part_ml, ws.splits, scale, ws.prefix,
                                 ws.chunk_cnt if _FUSED_COMBINE else None)
    return out


def sample_ref(logits: torch.Tensor, temperature: torch.Tensor, generator: torch.Generator | None = None,
               forced: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    lf = logits.float()
    t = temperature.float().to(lf.device)
    greedy = t <= 0
    scaled = lf / torch.where(greedy, torch.ones_like(t), t)[:, None]
    logp = torch.log_softmax(scaled, -1)
    probs = logp.exp()
    tok = torch.multinomial(probs, 1, generator=generator).squeeze(-1)
    tok = torch.where(greedy, scaled.argmax(-1), tok)
    if forced is not None:
        tok = torch.where(forced >= 0, forced.to(tok.device), tok)
    return tok, logp.gather(-1, tok[:, None]).squeeze(-1)


def sample(logits: torch.Tensor, temperature: torch.Tensor, seed: torch.Tensor, generator: torch.Generator | None = None,
           forced: torch.Tensor | None = None, row_ids: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Categorical sample per row at its temperature (<=0: greedy) with the token's log-prob.
    ``forced[row] >= 0`` overrides the token (its log-prob is still reported).
    ``row_ids`` names each row's random stream (stable across batch re-ordering)."""
    if not logits.is_cuda:
        return sample_ref(logits, temperature, generator, forced)
    B = logits.shape[0]
    tok = torch.empty(B, dtype=torch.int64, device=logits.device)
    lp = torch.empty(B, dtype=torch.float32, device=logits.device)
    _ext.ext().sample_tokens(logits, temperature, seed, tok, lp, row_ids, forced)
    return tok, lp


def sample_filtered(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor, min_p: torch.Tensor,
                    presence: torch.Tensor | None = None, frequency: torch.Tensor | None = None, repetition: torch.Tensor | None = None,
                    history: torch.Tensor | None = None, bias: torch.Tensor | None = None, forced: torch.Tensor | None = None,
                    generator: torch.Generator | None = None, kmax: int = 1024) -> tuple[torch.Tensor, torch.Tensor]:
    """Sampling with the full SGLang-style controls (fixed shapes: CUDA-graph capturable).

    Per row: repetition penalty (HF rule: divide positive / multiply negative logits of tokens seen),
    frequency and presence penalties over ``history`` (generated tokens, -1 = empty), additive
    ``bias`` (logit bias, or -inf outside an allowed set), temperature, then top-k, top-p (on the
    ``kmax`` best candidates) and min-p filtering and a Gumbel-max draw.  Temperature <= 0 is greedy.
    The reported log-prob is that of the sampled token under the temperature-scaled, unfiltered
    distribution — the quantity the trainer recomputes."""
    lf = logits.float()
    B, V = lf.shape
    greedy = temperature <= 0
    t = torch.where(greedy, torch.ones_like(temperature), temperature).float()[:, None]
    z = lf
    if history is not None:
        valid = (history >= 0).float()
        counts = torch.zeros_like(lf).scatter_add_(1, history.clamp(min=0).long(), valid)
        seen = counts > 0
        if repetition is not None:
            rp = repetition.float()[:, None]
            z = torch.where(seen, torch.where(z > 0, z / rp, z * rp), z)
        if frequency is not None:
            z = z - frequency.float()[:, None] * counts
        if presence is not None:
            z = z - presence.float()[:, None] * seen.float()
    if bias is not None:
        z = z + bias.float()
    z = z / t
    k = min(kmax, V)
    vals, idx = torch.topk(z, k, dim=-1)
    ar = torch.arange(k, device=lf.device)[None, :]
    k_eff = torch.where(top_k > 0, top_k, torch.full_like(top_k, k)).clamp(max=k)
    drop = ar >= k_eff[:, None]
    probs = torch.softmax(vals.masked_fill(drop, float("-inf")), -1)
    before = probs.cumsum(-1) - probs
    drop = drop | (before > top_p.float()[:, None])
    drop = drop | (probs < min_p.float()[:, None] * probs[:, :1])
    drop[:, 0] = False  # the best candidate always survives
    vals = vals.masked_fill(drop, float("-inf"))
    u = torch.rand(vals.shape, device=lf.device, generator=generator).clamp_(1e-20, 1.0)
    pick = torch.argmax(vals - torch.log(-torch.log(u)), -1)
    tok = torch.where(greedy, idx[:, 0], idx.gather(1, pick[:, None]).squeeze(1))
    if forced is not None:
        tok = torch.where(forced >= 0, forced.to(tok.dtype), tok)
    scaled = lf / t
    lp = scaled.gather(1, tok[:, None]).squeeze(1) - torch.logsumexp(scaled, -1)
    return tok, lp
