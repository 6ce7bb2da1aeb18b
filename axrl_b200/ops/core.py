"""Autograd-aware hot ops.

CUDA tensors run the sm_100a kernels in ``axrl_b200/csrc`` (loaded through
:mod:`axrl_b200.ops._ext`, which raises when the extension is missing).  CPU
tensors run the PyTorch definitions below, which double as the numerical
oracle for the GPU tests.

Op                 | reference call site it replaces
-------------------|-----------------------------------------------------------
rms_norm           | TE fused RMSNorm inside Megatron layers
qk_norm_rope       | TE fused RoPE (``axrl/utils/megatron/magi_forward.py:405-430``) + Qwen3 q/k norm
swiglu             | Megatron/TE gated activation
attention          | TE FA3 THD varlen / MagiAttention FFA (``magi_forward.py:445-466``)
linear             | TE / cuBLAS dense GEMMs
"""

from __future__ import annotations

import math

import torch

from axrl_b200.ops import _ext
from axrl_b200.ops.attention_spec import AttnSpec, dense_mask

# ----------------------------------------------------------------------------- RMSNorm


def _to_main_grad(w: torch.Tensor, dw: torch.Tensor):  # noqa: ANN202
    """Weight gradient of a small parameter: added into its fp32 ``main_grad`` when the optimizer
    attached one (so every gradient is final when the layer's backward ends), else returned."""
    main = getattr(w, "main_grad", None)
    if main is not None:
        main.add_(dw.float())
        return None
    return dw.to(w.dtype)


def _rms_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):  # noqa: ANN001, ANN205
        y, rstd = _ext.ext().rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x, w, rstd = ctx.saved_tensors
        dx, dw = _ext.ext().rmsnorm_bwd(dy.contiguous(), x, w, rstd)
        return dx, _to_main_grad(w, dw), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if not x.is_cuda:
        return _rms_ref(x, w, eps)
    shp = x.shape
    return _RMSNorm.apply(x.reshape(-1, shp[-1]).contiguous(), w, eps).view(shp)


# ----------------------------------------------------------------------------- q/k norm + RoPE


def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:  # noqa: ANN001
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))


def _rope_ref(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    # x: (T, H, D); neox-style rotate-half over the first 2 * len(inv_freq) dims (all of them unless the
    # rotary embedding is partial), the remaining dims passed through; angles in fp32.
    R = 2 * inv_freq.numel()
    ang = pos.float()[:, None] * inv_freq[None, :].to(pos.device)
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    xf = x.float()
    xr = xf[..., :R]
    h = R // 2
    rot = torch.cat([-xr[..., h:], xr[..., :h]], -1)
    out = xr * cos + rot * sin
    if R < xf.shape[-1]:
        out = torch.cat([out, xf[..., R:]], -1)
    return out.to(x.dtype)


def _qk_norm_rope_ref(qkv, qw, kw, pos, inv_freq, nq, nkv, eps):  # noqa: ANN001, ANN202
    T = qkv.shape[0]
    D = qw.numel()
    q, k, v = qkv.view(T, nq + 2 * nkv, D).split([nq, nkv, nkv], dim=1)
    q = _rope_ref(_rms_ref(q, qw, eps), pos, inv_freq)
    k = _rope_ref(_rms_ref(k, kw, eps), pos, inv_freq)
    return q.contiguous(), k.contiguous(), v.contiguous()


def check_full_rotary(qw: torch.Tensor, inv_freq: torch.Tensor) -> None:
    """The q/k-norm + RoPE kernels rotate the whole head (head_dim 128)."""
    if 2 * inv_freq.numel() != qw.numel():
        raise NotImplementedError(f"partial rotary embedding ({2 * inv_freq.numel()} of {qw.numel()} dims) has no CUDA kernel yet")


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, pos, inv_freq, nq, nkv, eps):  # noqa: ANN001, ANN205
        q, k, v, rstd = _ext.ext().qknorm_rope_fwd(qkv, qw, kw, pos, inv_freq, nq, nkv, eps)
        ctx.save_for_backward(qkv, qw, kw, pos, inv_freq, rstd)
        ctx.shape = (nq, nkv)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):  # noqa: ANN001, ANN205
        qkv, qw, kw, pos, inv_freq, rstd = ctx.saved_tensors
        nq, nkv = ctx.shape
        dqkv, dqw, dkw = _ext.ext().qknorm_rope_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), qkv, qw, kw, pos, inv_freq, rstd, nq, nkv)
        return dqkv, _to_main_grad(qw, dqw), _to_main_grad(kw, dkw), None, None, None, None, None


def qk_norm_rope(qkv, q_norm_w, k_norm_w, pos, inv_freq, nq: int, nkv: int, eps: float = 1e-6):  # noqa: ANN001, ANN201
    """Split fused QKV rows, RMS-normalise q/k per head, apply RoPE at ``pos``.
    Returns contiguous ``q (T,nq,D)``, ``k (T,nkv,D)``, ``v (T,nkv,D)``."""
    if not qkv.is_cuda:
        return _qk_norm_rope_ref(qkv, q_norm_w, k_norm_w, pos, inv_freq, nq, nkv, eps)
    check_full_rotary(q_norm_w, inv_freq)
    return _QKNormRope.apply(qkv.contiguous(), q_norm_w, k_norm_w, pos.to(torch.int32).contiguous(), inv_freq, nq, nkv, eps)


# ----------------------------------------------------------------------------- SwiGLU


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):  # noqa: ANN001, ANN205
        ctx.save_for_backward(gu)
        return _ext.ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (gu,) = ctx.saved_tensors
        return _ext.ext().swiglu_bwd(dy.contiguous(), gu)


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` where each row is ``[gate | up]``."""
    if not gate_up.is_cuda:
        g, u = gate_up.float().chunk(2, -1)
        return (torch.nn.functional.silu(g) * u).to(gate_up.dtype)
    return _SwiGLU.apply(gate_up.contiguous())


# ----------------------------------------------------------------------------- attention


def _attn_ref(q, k, v, spec: AttnSpec, scale: float):  # noqa: ANN001, ANN202
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    mask = dense_mask(spec).to(q.device)
    kk = k.float().repeat_interleave(rep, 1)
    vv = v.float().repeat_interleave(rep, 1)
    s = torch.einsum("thd,shd->hts", q.float(), kk) * scale
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    return torch.einsum("hts,shd->thd", p, vv).to(q.dtype)


class AttnStash:
    """Attention outputs (o, lse) of a checkpointed layer's first forward, reused by the forward
    that backward replays, so activation recompute re-runs the projections and norms but not the
    attention kernel (o and lse of one layer are (T, Hq, D) bf16 + (T, Hq) fp32).  The first
    forward pushes, the replay pops the entry of the same spec and shape (FIFO per key, which is
    the backward order of micro-batches under 1F1B and interleaved schedules)."""

    pushing = False  # set (by the model) around the first forward of checkpointed layers

    def __init__(self) -> None:
        self.items: dict[tuple, list[tuple[torch.Tensor, torch.Tensor]]] = {}

    def clear(self) -> None:
        self.items.clear()


class _Attn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, spec, scale, stash=None):  # noqa: ANN001, ANN205
        key = (id(spec), tuple(q.shape))
        hit = None
        if stash is not None and not AttnStash.pushing:
            lst = stash.items.get(key)
            if lst:
                hit = lst.pop(0)
                if not lst:
                    del stash.items[key]
        if hit is not None:
            o, lse = hit
        else:
            o, lse = _ext.ext().attn_fwd(q, k, v, spec.qseg, spec.kr, spec.fwd_tiles, scale)
            if stash is not None and AttnStash.pushing:
                stash.items.setdefault(key, []).append((o, lse))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.spec, ctx.scale = spec, scale
        return o

    @staticmethod
    def backward(ctx, do):  # noqa: ANN001, ANN205
        q, k, v, o, lse = ctx.saved_tensors
        s = ctx.spec
        dq, dk, dv = _ext.ext().attn_bwd(do.contiguous(), q, k, v, o, lse, s.kseg, s.qr, s.bwd_tiles, ctx.scale, s.bwd_tiles_tc,
                                         s.qseg, s.kr, s.fwd_tiles)
        return dq, dk, dv, None, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: AttnSpec, scale: float | None = None,
              stash: AttnStash | None = None) -> torch.Tensor:
    """Range-list attention over packed tokens.  q: (T,Hq,D); k,v: (T,Hkv,D) with GQA."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if not q.is_cuda:
        return _attn_ref(q, k, v, spec, scale)
    if not spec.qseg.is_cuda:
        spec = spec.to(q.device)
    return _Attn.apply(q.contiguous(), k.contiguous(), v.contiguous(), spec, scale, stash)


# ------------------------------------------------------- split-key attention (ring / context parallel)
# The keys of one query set split over sources s (context-parallel ranks): each source gives a
# partial (o_s, lse2_s) — lse2 in the log2 domain, (Hq, T), +inf for a row with no keys there —
# and the merge weights o_s by 2^(lse2_s - lse2).  The backward of every source uses the final
# (o, lse2): its probabilities 2^(S*scale*log2e - lse2) are the rows of the full softmax.

_LOG2E = 1.4426950408889634


def _part_probs(q, k, spec, scale, lse2):  # noqa: ANN001, ANN202
    rep = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1)
    s2 = torch.einsum("thd,shd->hts", q.float(), kk) * (scale * _LOG2E)
    mask = dense_mask(spec).to(q.device)[None]
    if lse2 is None:
        m = s2.masked_fill(~mask, float("-inf")).amax(-1, keepdim=True)
        l = torch.exp2(s2 - m.clamp_min(-1e30)).masked_fill(~mask, 0.0).sum(-1)
        lse2 = torch.where(l > 0, m.squeeze(-1) + torch.log2(l.clamp_min(1e-30)), torch.full_like(l, float("inf")))
    p = torch.exp2(s2 - lse2[..., None]).masked_fill(~mask, 0.0)
    return p, lse2


def attn_partial(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: AttnSpec, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(o, lse2) of the queries against one key source (no autograd)."""
    if q.is_cuda:
        if not spec.qseg.is_cuda:
            spec = spec.to(q.device)
        o, lse2 = _ext.ext().attn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), spec.qseg, spec.kr, spec.fwd_tiles, scale)
        return o, lse2
    p, lse2 = _part_probs(q, k, spec, scale, None)
    rep = q.shape[1] // k.shape[1]
    o = torch.einsum("hts,shd->thd", p, v.float().repeat_interleave(rep, 1))
    return o.to(q.dtype), lse2.contiguous()


def attn_merge(parts: list[tuple[torch.Tensor, torch.Tensor]]) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge per-source partials into (o, lse2)."""
    if parts[0][0].is_cuda:
        o, lse2 = _ext.ext().attn_merge([p[0] for p in parts], [p[1] for p in parts])
        return o, lse2
    lse = torch.stack([p[1] for p in parts])
    fin = torch.where(torch.isinf(lse) & (lse > 0), torch.full_like(lse, float("-inf")), lse)
    m = fin.amax(0)
    w = torch.exp2(fin - m.clamp_min(-1e30)[None])
    den = w.sum(0)
    o = sum(p[0].float() * (w[i] / den.clamp_min(1e-30)).t()[..., None] for i, p in enumerate(parts))
    lse2 = torch.where(den > 0, m + torch.log2(den.clamp_min(1e-30)), torch.full_like(den, float("inf")))
    return o.to(parts[0][0].dtype), lse2


def attn_bwd_dsum(o: torch.Tensor, do: torch.Tensor) -> torch.Tensor:
    """rowsum(dO * O) as (Hq, T) fp32."""
    if o.is_cuda:
        return _ext.ext().attn_bwd_dsum(o.contiguous(), do.contiguous())
    return (o.float() * do.float()).sum(-1).t().contiguous()


def attn_bwd_partial(do: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lse2: torch.Tensor, dsum: torch.Tensor,
                     dq_acc: torch.Tensor, spec: AttnSpec, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(dK, dV) of one key source; its share of dQ is added into ``dq_acc`` (fp32)."""
    if q.is_cuda:
        if not spec.qseg.is_cuda:
            spec = spec.to(q.device)
        dk, dv = _ext.ext().attn_bwd_partial(do.contiguous(), q, k.contiguous(), v.contiguous(), lse2, dsum, dq_acc, spec.kseg, spec.qr,
                                             spec.bwd_tiles, scale, spec.bwd_tiles_tc)
        return dk, dv
    Hkv = k.shape[1]
    rep = q.shape[1] // Hkv
    p, _ = _part_probs(q, k, spec, scale, lse2)
    dof = do.float()
    dp = torch.einsum("thd,shd->hts", dof, v.float().repeat_interleave(rep, 1))
    ds = p * (dp - dsum[..., None])
    dq_acc += torch.einsum("hts,shd->thd", ds, k.float().repeat_interleave(rep, 1)) * scale
    dk = torch.einsum("hts,thd->shd", ds, q.float()) * scale
    dv = torch.einsum("hts,thd->shd", p, dof)
    S = k.shape[0]
    return (dk.view(S, Hkv, rep, -1).sum(2).to(k.dtype), dv.view(S, Hkv, rep, -1).sum(2).to(v.dtype))


# ----------------------------------------------------------------------------- linear


def _gemm(a: torch.Tensor, b: torch.Tensor, trans_b: bool) -> torch.Tensor:
    return _ext.ext().gemm(a, b, trans_b)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):  # noqa: ANN001, ANN205
        ctx.save_for_backward(x, w)
        return _ext.ext().linear_fwd(x, w)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        e = _ext.ext()
        dx = e.linear_dgrad(dy, w) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                e.linear_wgrad_acc(dy, x, main)  # fp32 accumulate in place
                dw = None
            else:
                dw = e.linear_wgrad(dy, x)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` for x (..., K), w (N, K).  On GPU the weight grad accumulates
    straight into ``w.main_grad`` (fp32) when present."""
    if not x.is_cuda:
        return torch.nn.functional.linear(x, w)
    shp = x.shape
    y = _Linear.apply(x.reshape(-1, shp[-1]).contiguous(), w)
    return y.view(*shp[:-1], w.shape[0])


# ----------------------------------------------------------------------------- embedding


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table):  # noqa: ANN001, ANN205
        ctx.save_for_backward(ids)
        ctx.table = table
        return _ext.ext().embed_fwd(ids, table)

    @staticmethod
    def backward(ctx, dout):  # noqa: ANN001, ANN205
        (ids,) = ctx.saved_tensors
        table = ctx.table
        main = getattr(table, "main_grad", None)
        if main is not None:
            _ext.ext().embed_bwd(ids, dout.contiguous(), main)
            return None, None
        g = torch.zeros(table.shape, dtype=torch.float32, device=table.device)
        _ext.ext().embed_bwd(ids, dout.contiguous(), g)
        return None, g.to(table.dtype)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Row gather; on GPU the backward scatter-adds into ``table.main_grad`` (fp32)."""
    if not table.is_cuda:
        return torch.nn.functional.embedding(ids.long(), table)
    return _Embed.apply(ids.long().contiguous(), table)
