"""Gated DeltaNet (GDN) token mixer for hybrid linear / full-attention decoders (Qwen3-Next / 3.5 style).

Reference: the GDN branch of the reference's packed forward (``axrl/utils/megatron/magi_forward.py:790-848``,
Megatron's ``experimental_attention_variant="gated_delta_net"``; its kernels come from
flash-linear-attention).  Per value head, with state ``S`` (d_k x d_v) and token ``t``::

    a_t = exp(g_t)                                   g_t = -exp(A_log) * softplus(a_t + dt_bias)
    S_t = a_t S_{t-1} + beta_t k_t (v_t - a_t S_{t-1}^T k_t)^T          beta_t = sigmoid(b_t)
    o_t = S_t^T q_t / sqrt(d_k)

q, k, v first pass a causal depthwise convolution (kernel 4) + SiLU, and q, k are L2-normalised
(key heads are shared by ``num_v / num_k`` value heads).  The head outputs are RMS-normalised,
gated by SiLU(z) and projected back to the hidden size.

Training / prefill use the chunked form (chunk C): with G the within-chunk cumulative sum of g,
A_tj = -beta_t exp(G_t - G_j) k_t.k_j (j < t), T = (I - A)^-1, W = T diag(beta e^G) K and
U = T diag(beta) V, a chunk entered with state S_0 has

    D      = U - W S_0                               (the corrected values)
    O      = diag(e^G) Q S_0 + ((Q K^T) o M) D       M_tj = exp(G_t - G_j), j <= t
    S_next = e^{G_C} S_0 + (K o e^{G_C - G})^T D

so each chunk costs a few (C x d) matmuls and one triangular solve; the recurrence runs over
chunks.  Decode advances the recurrent state one token at a time.  Sequences are independent:
the state starts at zero at every packed sequence start.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn


def _segments(spec, T: int) -> list[tuple[int, int]]:  # noqa: ANN001
    """Packed sequences of a flat causal spec (one causal range per sequence)."""
    out = []
    for q0, q1, a, b in spec.qseg.cpu().tolist():
        rng = spec.kr[a:b].cpu().tolist()
        if len(rng) != 1 or rng[0][0] != q0 or rng[0][2] != 1:
            raise ValueError("GDN layers need flat causal packing (prefix-tree merged samples are not supported)")
        out.append((q0, q1))
    return out


def causal_conv(x: torch.Tensor, w: torch.Tensor, starts: torch.Tensor) -> torch.Tensor:
    """Depthwise causal convolution over packed tokens + SiLU.  x (T, C), w (C, K); ``starts`` (T,)
    holds each token's offset inside its sequence (no tap reaches into the previous sequence)."""
    K = w.shape[1]
    out = x * w[:, K - 1]
    for j in range(1, K):
        sh = torch.zeros_like(x)
        sh[j:] = x[:-j]
        sh = sh * (starts >= j).to(x.dtype)[:, None]
        out = out + sh * w[:, K - 1 - j]
    return F.silu(out)


def gated_delta_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                        state: torch.Tensor | None = None, chunk: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """One sequence: q, k (L, H, dk) (normalised, q pre-scaled), v (L, H, dv), g, beta (L, H), fp32.
    Returns o (L, H, dv) and the final state (H, dk, dv)."""
    L, H, dk = k.shape
    dv = v.shape[-1]
    S = torch.zeros(H, dk, dv, dtype=torch.float32, device=q.device) if state is None else state.float().clone()
    pad = (-L) % chunk
    if pad:
        zq = lambda t: torch.cat([t, t.new_zeros((pad,) + t.shape[1:])])  # noqa: E731
        q, k, v, g, beta = zq(q), zq(k), zq(v), zq(g), zq(beta)
    n = (L + pad) // chunk
    # (H, n, C, .)
    Q, Kc, Vc = (t.reshape(n, chunk, H, -1).permute(2, 0, 1, 3) for t in (q, k, v))
    Gs = g.reshape(n, chunk, H).permute(2, 0, 1).cumsum(-1)
    B = beta.reshape(n, chunk, H).permute(2, 0, 1)
    diff = Gs[..., :, None] - Gs[..., None, :]  # G_t - G_j
    lower = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device))
    strict = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device), -1)
    decay = torch.where(lower, diff, torch.full_like(diff, -torch.inf)).exp()  # M (inclusive)
    kk = Kc @ Kc.transpose(-1, -2)
    A = torch.where(strict, -(B[..., :, None] * decay * kk), torch.zeros_like(kk))
    eye = torch.eye(chunk, dtype=torch.float32, device=q.device)
    Tm = torch.linalg.solve_triangular(eye - A, eye.expand_as(A).contiguous(), upper=False, unitriangular=True)
    W = Tm @ (Kc * (B * Gs.exp())[..., None])
    U = Tm @ (Vc * B[..., None])
    qk = (Q @ Kc.transpose(-1, -2)) * decay
    eG = Gs.exp()
    tail = (Gs[..., -1:] - Gs).exp()  # exp(G_C - G_j)
    outs = []
    for c in range(n):
        Dc = U[:, c] - W[:, c] @ S
        outs.append((Q[:, c] * eG[:, c, :, None]) @ S + qk[:, c] @ Dc)
        S = eG[:, c, -1, None, None] * S + (Kc[:, c] * tail[:, c, :, None]).transpose(-1, -2) @ Dc
    o = torch.stack(outs, 1).reshape(H, n * chunk, dv).transpose(0, 1)[:L]
    return o, S


def gated_delta_chunked_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                               segs: list[tuple[int, int]], chunk: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`gated_delta_chunked` over every packed sequence at once.

    q, k (T, H, dk), v (T, H, dv), g, beta (T, H) fp32; ``segs`` the sequences' (start, end).  The
    within-chunk algebra (decay masks, the triangular solve, W, U, Q K^T) runs batched over all
    chunks of all sequences; the state recurrence then advances every sequence that still has a
    chunk left, one chunk position per step (as many steps as the longest sequence has chunks).
    A sequence's last chunk is padded with g = 0, beta = 0, k = v = 0, which leaves its state as it
    was.  Returns o (T, H, dv) and the final states (len(segs), H, dk, dv)."""
    T, H, dk = k.shape
    dv = v.shape[-1]
    dev = q.device
    C = chunk
    rows, steps = [], []  # token index of each chunk slot (-1 = padding); per sequence its chunk ids
    for s0, s1 in segs:
        ids = []
        for c0 in range(s0, s1, C):
            r = list(range(c0, min(c0 + C, s1)))
            ids.append(len(rows))
            rows.append(r + [-1] * (C - len(r)))
        steps.append(ids)
    B = len(segs)
    if not rows:
        return q.new_zeros(T, H, dv), q.new_zeros(B, H, dk, dv)
    idx = torch.tensor(rows, dtype=torch.long, device=dev)  # (M, C)
    valid = idx >= 0
    src = idx.clamp(min=0)
    vm = valid[..., None].float()

    def take(x: torch.Tensor) -> torch.Tensor:  # (T, H, d) -> (M, H, C, d), zero on padding
        return (x[src] * vm[..., None]).permute(0, 2, 1, 3)

    Q, Kc, Vc = take(q), take(k), take(v)
    Gs = (g[src] * vm).permute(0, 2, 1).cumsum(-1)  # (M, H, C)
    Bt = (beta[src] * vm).permute(0, 2, 1)
    diff = Gs[..., :, None] - Gs[..., None, :]
    lower = torch.tril(torch.ones(C, C, dtype=torch.bool, device=dev))
    strict = torch.tril(torch.ones(C, C, dtype=torch.bool, device=dev), -1)
    decay = torch.where(lower, diff, torch.full_like(diff, -torch.inf)).exp()
    kk = Kc @ Kc.transpose(-1, -2)
    A = torch.where(strict, -(Bt[..., :, None] * decay * kk), torch.zeros_like(kk))
    eye = torch.eye(C, dtype=torch.float32, device=dev)
    Tm = torch.linalg.solve_triangular(eye - A, eye.expand_as(A).contiguous(), upper=False, unitriangular=True)
    eG = Gs.exp()
    W = Tm @ (Kc * (Bt * eG)[..., None])
    U = Tm @ (Vc * Bt[..., None])
    qk = (Q @ Kc.transpose(-1, -2)) * decay
    Kt = (Kc * (Gs[..., -1:] - Gs).exp()[..., None]).transpose(-1, -2)  # (K o e^{G_C - G})^T
    S = q.new_zeros(B, H, dk, dv)
    outs, out_ids = [], []
    for c in range(max(len(s) for s in steps)):
        act = [i for i, s in enumerate(steps) if len(s) > c]
        a = torch.tensor(act, dtype=torch.long, device=dev)
        m = torch.tensor([steps[i][c] for i in act], dtype=torch.long, device=dev)
        Sa = S.index_select(0, a)
        D = U.index_select(0, m) - W.index_select(0, m) @ Sa
        outs.append((Q.index_select(0, m) * eG.index_select(0, m)[..., None]) @ Sa + qk.index_select(0, m) @ D)
        out_ids.append(m)
        Sn = eG.index_select(0, m)[:, :, -1, None, None] * Sa + Kt.index_select(0, m) @ D
        S = S.index_copy(0, a, Sn)
    O = torch.cat(outs).new_zeros(idx.shape[0], H, C, dv).index_copy(0, torch.cat(out_ids), torch.cat(outs))
    flat = O.permute(0, 2, 1, 3).reshape(-1, H, dv)[valid.reshape(-1)]
    o = q.new_zeros(T, H, dv).index_copy(0, idx.reshape(-1)[valid.reshape(-1)], flat)
    return o, S


def gated_delta_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                     S: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """One token for a batch: q, k (B, H, dk), v (B, H, dv), g, beta (B, H), S (B, H, dk, dv) fp32."""
    S = S * g.exp()[..., None, None]
    delta = beta[..., None] * (v - (S * k[..., None]).sum(-2))
    S = S + k[..., None] * delta[..., None, :]
    return (S * q[..., None]).sum(-2), S


def gated_delta_recurrent(q, k, v, g, beta, state=None):  # noqa: ANN001, ANN201
    """Token-by-token reference of :func:`gated_delta_chunked` (tests)."""
    L, H, dk = k.shape
    S = torch.zeros(1, H, dk, v.shape[-1], dtype=torch.float32, device=q.device) if state is None else state[None].float()
    outs = []
    for t in range(L):
        o, S = gated_delta_step(q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1], beta[t:t + 1], S)
        outs.append(o)
    return torch.cat(outs), S[0]


class GatedDeltaNet(nn.Module):
    """Under tensor parallelism (``tp_size`` ranks) each rank holds 1/tp of the key and value heads
    (value head j reads key head j // (nv / nk), so contiguous head blocks stay together): the q/k/v,
    z, b, a projections, the convolution channels, ``dt_bias`` and ``A_log`` are split by heads, the
    output projection by its input columns; the recurrence then runs on whole sequences of this
    rank's heads (the sequence-parallel input is all-gathered once, the output reduce-scattered),
    as Megatron shards its GDN layers."""

    def __init__(self, cfg, tp_size: int = 1) -> None:  # noqa: ANN001
        super().__init__()
        H = cfg.hidden_size
        if cfg.linear_num_key_heads % tp_size or cfg.linear_num_value_heads % tp_size:
            raise ValueError("linear-attention key / value heads must split evenly over TP ranks")
        self.nk, self.nv = cfg.linear_num_key_heads // tp_size, cfg.linear_num_value_heads // tp_size
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.kernel = cfg.linear_conv_kernel_dim
        self.eps = cfg.rms_norm_eps
        self.key_dim, self.value_dim = self.nk * self.dk, self.nv * self.dv
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.in_proj_qkv = nn.Parameter(torch.empty(self.conv_dim, H))
        self.in_proj_z = nn.Parameter(torch.empty(self.value_dim, H))
        self.in_proj_b = nn.Parameter(torch.empty(self.nv, H))
        self.in_proj_a = nn.Parameter(torch.empty(self.nv, H))
        self.conv_weight = nn.Parameter(torch.empty(self.conv_dim, self.kernel))
        self.dt_bias = nn.Parameter(torch.ones(self.nv))
        self.A_log = nn.Parameter(torch.ones(self.nv))
        self.norm_weight = nn.Parameter(torch.ones(self.dv))
        self.out_proj = nn.Parameter(torch.empty(H, self.value_dim))
        self.cp = None

    # ---- shared pieces
    def _project(self, x: torch.Tensor):  # noqa: ANN202
        mixed = F.linear(x, self.in_proj_qkv)
        z = F.linear(x, self.in_proj_z)
        b = F.linear(x, self.in_proj_b).float()
        a = F.linear(x, self.in_proj_a).float()
        return mixed, z, b, a

    def _heads(self, mixed: torch.Tensor, b: torch.Tensor, a: torch.Tensor, heads: tuple | None = None):  # noqa: ANN202
        """``heads`` = (nk, nv, A_log, dt_bias) of a head subset (context parallelism); default all."""
        nk, nv, A_log, dt_bias = heads or (self.nk, self.nv, self.A_log, self.dt_bias)
        T = mixed.shape[0]
        q, k, v = torch.split(mixed.float(), [nk * self.dk, nk * self.dk, nv * self.dv], -1)
        q = q.reshape(T, nk, self.dk)
        k = k.reshape(T, nk, self.dk)
        v = v.reshape(T, nv, self.dv)
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
        rep = nv // nk
        if rep > 1:
            q, k = q.repeat_interleave(rep, 1), k.repeat_interleave(rep, 1)
        q = q / math.sqrt(self.dk)
        g = -A_log.float().exp() * F.softplus(a + dt_bias.float())
        return q, k, v, g, b.sigmoid()

    def _forward_cp(self, mixed: torch.Tensor, b: torch.Tensor, a: torch.Tensor, layout) -> torch.Tensor:  # noqa: ANN001
        """Context parallelism: every rank holds a zigzag slice of each sequence.  An all-to-all swaps
        the sequence split for a head split (rank j gets every token of head group j), the recurrence
        runs on whole sequences, and a second all-to-all returns the outputs to the token owners."""
        from axrl_b200.parallel.context_parallel import heads_to_seq, seq_to_heads

        cp = self.cp
        P, j, L = cp.size, cp.rank, mixed.shape[0]
        if self.nk % P:
            raise ValueError("linear-attention key heads must split evenly over context-parallel ranks")
        nkg, nvg = self.nk // P, self.nv // P
        q, k, v = torch.split(mixed.float(), [self.key_dim, self.key_dim, self.value_dim], -1)
        groups = torch.cat([q.reshape(L, P, -1), k.reshape(L, P, -1), v.reshape(L, P, -1), b.reshape(L, P, nvg),
                            a.reshape(L, P, nvg)], -1)  # (L, P, channels of one head group)
        xg = seq_to_heads(groups.float(), cp)  # (P*L, .) rank-major stream, head group j
        perm = layout.perm.to(xg.device)
        xs = xg.index_select(0, perm)  # sequence order
        kd, vd = nkg * self.dk, nvg * self.dv
        m_g, b_g, a_g = torch.split(xs, [2 * kd + vd, nvg, nvg], -1)
        wq, wk, wv = torch.split(self.conv_weight, [self.key_dim, self.key_dim, self.value_dim], 0)
        w_g = torch.cat([wq.reshape(P, kd, -1)[j], wk.reshape(P, kd, -1)[j], wv.reshape(P, vd, -1)[j]], 0)
        T = xs.shape[0]
        starts = torch.zeros(T, dtype=torch.long, device=xs.device)
        for s0, s1 in layout.segs:
            starts[s0:s1] = torch.arange(s1 - s0, device=xs.device)
        conv = causal_conv(m_g, w_g.float(), starts)
        sl = slice(j * nvg, (j + 1) * nvg)
        qh, kh, vh, g, beta = self._heads(conv, b_g, a_g, (nkg, nvg, self.A_log[sl], self.dt_bias[sl]))
        o = gated_delta_chunked_varlen(qh, kh, vh, g, beta, layout.segs)[0]
        o_stream = torch.empty_like(o).index_copy(0, perm, o)  # back to the rank-major stream
        return heads_to_seq(o_stream.reshape(T, vd), cp).reshape(L, self.nv, self.dv)

    def _out(self, o: torch.Tensor, z: torch.Tensor, dtype: torch.dtype, tp=None) -> torch.Tensor:  # noqa: ANN001
        T = o.shape[0]
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + self.eps) * self.norm_weight.float()
        o = o * F.silu(z.float().reshape(T, self.nv, self.dv))
        o = o.reshape(T, self.value_dim).to(dtype)
        if tp is not None:
            from axrl_b200.parallel.tensor_parallel import row_parallel_linear

            return row_parallel_linear(o, self.out_proj, tp)
        return F.linear(o, self.out_proj)

    # ---- training / prefill over packed sequences
    def forward(self, x: torch.Tensor, pos, inv_freq, spec, tp=None, states: list | None = None) -> torch.Tensor:  # noqa: ANN001
        """``states`` (optional, prefill): receives one (conv_state, recurrent_state) per sequence."""
        tp = tp if tp is not None and getattr(tp, "enabled", False) else None
        if tp is not None:  # whole sequences of this rank's heads: gather the sequence-parallel rows
            from axrl_b200.parallel.tensor_parallel import gather_from_sp

            x = gather_from_sp(x, tp)
        T = x.shape[0]
        layout = getattr(spec, "seq_layout", None)
        if self.cp is not None and getattr(self.cp, "enabled", False):
            if layout is None or states is not None:
                raise ValueError("Gated DeltaNet under context parallelism needs the CP packing's sequence layout")
            mixed, z, b, a = self._project(x)
            return self._out(self._forward_cp(mixed, b, a, layout), z, x.dtype, tp)
        segs = _segments(spec, T)
        starts = torch.zeros(T, dtype=torch.long, device=x.device)
        for s0, s1 in segs:
            starts[s0:s1] = torch.arange(s1 - s0, device=x.device)
        mixed, z, b, a = self._project(x)
        conv = causal_conv(mixed.float(), self.conv_weight.float(), starts)
        q, k, v, g, beta = self._heads(conv, b, a)
        o, S_all = gated_delta_chunked_varlen(q, k, v, g, beta, segs)
        if states is not None:
            for i, (s0, s1) in enumerate(segs):
                tailx = mixed[max(s0, s1 - (self.kernel - 1)):s1].float()
                cs = torch.zeros(self.kernel - 1, self.conv_dim, dtype=torch.float32, device=x.device)
                cs[cs.shape[0] - tailx.shape[0]:] = tailx
                states.append((cs, S_all[i]))
        return self._out(o, z, x.dtype, tp)

    # ---- decode: one token per row with carried states
    def step(self, x: torch.Tensor, conv_state: torch.Tensor, S: torch.Tensor) -> torch.Tensor:
        """x (B, H); conv_state (B, kernel-1, conv_dim) and S (B, nv, dk, dv) fp32, updated in place."""
        mixed, z, b, a = self._project(x)
        window = torch.cat([conv_state, mixed.float()[:, None]], 1)  # (B, kernel, C)
        conv = F.silu((window * self.conv_weight.float().t()[None]).sum(1))
        conv_state.copy_(window[:, 1:])
        q, k, v, g, beta = self._heads(conv, b, a)
        o, S_new = gated_delta_step(q, k, v, g, beta, S)
        S.copy_(S_new)
        return self._out(o, z, x.dtype)

    def step_pool(self, x: torch.Tensor, conv_pool: torch.Tensor, S_pool: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        """:meth:`step` on states kept in pools (rows ``slots``), the recurrent update done in place
        by the ``gdn_step`` kernel (csrc/kernels/gdn.cu) without gathering the states."""
        from axrl_b200.ops import _ext

        mixed, z, b, a = self._project(x)
        conv_state = conv_pool.index_select(0, slots)
        window = torch.cat([conv_state, mixed.float()[:, None]], 1)
        conv = F.silu((window * self.conv_weight.float().t()[None]).sum(1))
        conv_pool.index_copy_(0, slots, window[:, 1:])
        q, k, v, g, beta = self._heads(conv, b, a)
        o = _ext.ext().gdn_step(q.contiguous(), k.contiguous(), v.contiguous(), g.contiguous(), beta.contiguous(), S_pool, slots)
        return self._out(o, z, x.dtype)

