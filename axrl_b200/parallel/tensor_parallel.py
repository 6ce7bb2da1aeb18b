"""Tensor + sequence parallelism for the trainer (Megatron TP with ``sequence_parallel=True``).

Reference: ``MegatronWorkerConfig.tp_size`` (``axrl/configs.py:378``) and
``provider.sequence_parallel = tp > 1`` (``axrl/worker/megatron_worker.py:825``); Megatron's
Column/RowParallelLinear with SP, ``VocabParallelEmbedding`` and the vocab-parallel
log-prob / entropy of ``axrl/utils/megatron/tensor_parallel.py:8-82``.

Layout.  Between transformer blocks the hidden stream is split along tokens: TP rank ``r``
holds rows ``[r*T/tp, (r+1)*T/tp)`` of the packed micro-batch (every TP rank receives the
same micro-batch).  A block enters tensor parallelism with an all-gather of its normalised
input (column-parallel QKV / gate-up on the local heads / FFN columns) and leaves it with a
reduce-scatter of the partial output of the row-parallel O / down projection.  Embedding and
LM head are split over the vocabulary.  Norm weights (and any parameter that is replicated
across TP ranks) receive partial gradients and are all-reduced over the TP group before the
optimizer step (:func:`allreduce_replicated_grads`).

Communication goes through a :class:`TPComm`; :class:`TorchTPComm` (NCCL or gloo collectives)
is the reference path, :class:`axrl_b200.parallel.tp_overlap.P2PTPComm` the NVLink path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist


class TPComm:
    """Row-wise collectives over a TP group (rows = tokens)."""

    size: int = 1
    rank: int = 0

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class TorchTPComm(TPComm):
    def __init__(self, group: Any) -> None:
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nccl = dist.get_backend(group) == "nccl"

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        if self.nccl:
            out = torch.empty((self.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x, group=self.group)
            return out
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x, group=self.group)
        return torch.cat(parts, 0)

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        n = x.shape[0] // self.size
        assert n * self.size == x.shape[0], "rows must divide by the TP size"
        if self.nccl:
            out = torch.empty((n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
            dist.reduce_scatter_tensor(out, x, group=self.group)
            return out
        y = x.clone()
        dist.all_reduce(y, group=self.group)
        return y[self.rank * n:(self.rank + 1) * n].contiguous()

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(x, group=self.group)
        return x


@dataclass
class TPContext:
    size: int = 1
    rank: int = 0
    comm: TPComm | None = None
    group: Any = None

    @property
    def enabled(self) -> bool:
        return self.size > 1

    @classmethod
    def from_group(cls, group: Any, backend: str = "torch") -> "TPContext":
        if group is None or dist.get_world_size(group) == 1:
            return cls()
        if backend == "p2p":
            from axrl_b200.parallel.tp_overlap import P2PTPComm

            comm: TPComm = P2PTPComm(group)
        else:
            comm = TorchTPComm(group)
        return cls(size=comm.size, rank=comm.rank, comm=comm, group=group)

    def shard_range(self, n: int) -> tuple[int, int]:
        per = n // self.size
        return self.rank * per, (self.rank + 1) * per


# ----------------------------------------------------------------------------- autograd glue


class _GatherFromSP(torch.autograd.Function):
    """(T/tp, H) -> (T, H); backward reduce-scatters the (partial) gradient."""

    @staticmethod
    def forward(ctx, x, comm):  # noqa: ANN001, ANN205
        ctx.comm = comm
        return comm.all_gather_rows(x)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return ctx.comm.reduce_scatter_rows(g), None


class _ReduceScatterToSP(torch.autograd.Function):
    """(T, H) partial sums -> (T/tp, H) reduced rows; backward all-gathers."""

    @staticmethod
    def forward(ctx, x, comm):  # noqa: ANN001, ANN205
        ctx.comm = comm
        return comm.reduce_scatter_rows(x)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return ctx.comm.all_gather_rows(g.contiguous()), None


def gather_from_sp(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return _GatherFromSP.apply(x, tp.comm) if tp.enabled else x


def reduce_scatter_to_sp(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return _ReduceScatterToSP.apply(x, tp.comm) if tp.enabled else x


def column_parallel_linear(x_sp: torch.Tensor, w: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """``AG(x) @ w_shard.T``: (T/tp, K) -> (T, N/tp)."""
    from axrl_b200.ops import core

    if tp.enabled and x_sp.is_cuda and hasattr(tp.comm, "ag_linear"):
        y = tp.comm.ag_linear(x_sp, w)
        if y is not None:
            return y
    return core.linear(gather_from_sp(x_sp, tp), w)


def row_parallel_linear(x: torch.Tensor, w: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """``RS(x @ w_shard.T)``: (T, K/tp) -> (T/tp, N)."""
    from axrl_b200.ops import core

    if tp.enabled and x.is_cuda and hasattr(tp.comm, "linear_rs"):
        y = tp.comm.linear_rs(x, w)
        if y is not None:
            return y
    return reduce_scatter_to_sp(core.linear(x, w), tp)


# ----------------------------------------------------------------------------- vocab parallel


class _VocabParallelEmbed(torch.autograd.Function):
    """Embedding rows [v0, v0 + Vs) on this rank; other tokens contribute zeros.  The partial
    (T, H) sums are reduce-scattered into the SP layout."""

    @staticmethod
    def forward(ctx, ids, table, v0, comm):  # noqa: ANN001, ANN205
        Vs = table.shape[0]
        local = ids - v0
        inside = (local >= 0) & (local < Vs)
        idx = torch.where(inside, local, torch.zeros_like(local))
        part = table[idx] * inside[:, None].to(table.dtype)
        ctx.save_for_backward(idx, inside)
        ctx.table, ctx.comm = table, comm
        return comm.reduce_scatter_rows(part)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        idx, inside = ctx.saved_tensors
        table = ctx.table
        gf = ctx.comm.all_gather_rows(g.contiguous()).float() * inside[:, None]
        main = getattr(table, "main_grad", None)
        if main is not None:
            main.index_add_(0, idx, gf)
            return None, None, None, None
        dt = torch.zeros(table.shape, dtype=torch.float32, device=table.device)
        dt.index_add_(0, idx, gf)
        return None, dt.to(table.dtype), None, None


def vocab_parallel_embedding(ids: torch.Tensor, table_shard: torch.Tensor, tp: TPContext) -> torch.Tensor:
    v0 = tp.rank * table_shard.shape[0]
    return _VocabParallelEmbed.apply(ids.long(), table_shard, v0, tp.comm)


def combine_vocab_stats(lse_r: torch.Tensor, lab_r: torch.Tensor, es_r: torch.Tensor | None, comm: TPComm):
    """Combine per-rank (lse, label logit or 0, E[s]) rows into global (lp, lse, entropy).

    ``lse = logsumexp_r lse_r``; ``lp = sum_r lab_r - lse``;
    ``E[s] = sum_r exp(lse_r - lse) E_r[s]``; ``entropy = lse - E[s]``."""
    k = 3 if es_r is not None else 2
    stats = torch.stack([lse_r, lab_r] + ([es_r] if es_r is not None else []), 1).contiguous()  # (T, k)
    allst = comm.all_gather_rows(stats[None]).view(comm.size, -1, k)
    lse = torch.logsumexp(allst[:, :, 0], 0)
    lp = allst[:, :, 1].sum(0) - lse
    ent = None
    if es_r is not None:
        w = torch.exp(allst[:, :, 0] - lse[None])
        ent = lse - (w * allst[:, :, 2]).sum(0)
    return lp, lse, ent


class _VocabParallelLogprobRef(torch.autograd.Function):
    """Torch implementation (CPU and oracle): full-T hidden (already gathered), vocab shard."""

    @staticmethod
    def forward(ctx, hidden, w, labels, temperature, compute_entropy, v0, comm):  # noqa: ANN001, ANN205
        z = torch.nn.functional.linear(hidden.float(), w.float()) / temperature
        Vs = w.shape[0]
        lse_r = torch.logsumexp(z, -1)
        loc = labels - v0
        inside = (loc >= 0) & (loc < Vs) & (labels >= 0)
        lab_r = torch.where(inside, z.gather(-1, loc.clamp(0, Vs - 1)[:, None]).squeeze(-1), torch.zeros_like(lse_r))
        es_r = (torch.softmax(z, -1) * z).sum(-1) if compute_entropy else None
        lp, lse, ent = combine_vocab_stats(lse_r, lab_r, es_r, comm)
        ctx.save_for_backward(hidden, w, labels, lse, ent if ent is not None else lse)
        ctx.cfg = (temperature, compute_entropy, v0)
        return lp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):  # noqa: ANN001, ANN205
        hidden, w, labels, lse, ent = ctx.saved_tensors
        temperature, compute_entropy, v0 = ctx.cfg
        z = torch.nn.functional.linear(hidden.float(), w.float()) / temperature
        p = torch.exp(z - lse[:, None])
        Vs = w.shape[0]
        valid = labels >= 0
        gl = torch.where(valid, g_lp if g_lp is not None else torch.zeros_like(lse), torch.zeros_like(lse))
        dz = -p * gl[:, None]
        loc = labels - v0
        inside = (loc >= 0) & (loc < Vs) & valid
        rows = torch.nonzero(inside).squeeze(-1)
        dz[rows, loc[rows]] += gl[rows]
        if compute_entropy and g_ent is not None:
            es = lse - ent
            dz -= g_ent[:, None] * p * (z - es[:, None])
        dz = dz / temperature
        dh = (dz @ w.float()).to(hidden.dtype)
        dw = (dz.t() @ hidden.float())
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.add_(dw)
            dw = None
        else:
            dw = dw.to(w.dtype)
        return dh, dw, None, None, None, None, None


def vocab_parallel_logprob(hidden_full: torch.Tensor, w_shard: torch.Tensor, labels: torch.Tensor, tp: TPContext,
                           temperature: float = 1.0, compute_entropy: bool = False):  # noqa: ANN201
    """log p(label) and entropy over a vocabulary split across TP ranks.

    ``hidden_full`` is the gathered (T, H) final hidden state; its gradient is this rank's
    partial sum (the SP gather's backward reduce-scatters it)."""
    v0 = tp.rank * w_shard.shape[0]
    if hidden_full.is_cuda:
        from axrl_b200.ops.logprob import fused_logprob_vocab_parallel

        return fused_logprob_vocab_parallel(hidden_full, w_shard, labels, v0, tp.comm, temperature, compute_entropy)
    return _VocabParallelLogprobRef.apply(hidden_full, w_shard, labels.long(), float(temperature), bool(compute_entropy), v0, tp.comm)


# ----------------------------------------------------------------------------- params


def mark_replicated(p: torch.nn.Parameter) -> None:
    """A parameter held in full by every TP rank whose gradient is a partial sum."""
    p.tp_replicated = True


def replicated_params(model: torch.nn.Module) -> list[torch.nn.Parameter]:
    return [p for p in model.parameters() if getattr(p, "tp_replicated", False)]


def allreduce_replicated_grads(model: torch.nn.Module, tp: TPContext) -> None:
    """Sum the partial gradients of TP-replicated parameters (norm weights) over the TP group,
    coalesced into one buffer."""
    if not tp.enabled:
        return
    ps = [p for p in replicated_params(model) if getattr(p, "main_grad", None) is not None]
    if not ps:
        return
    flat = torch.cat([p.main_grad.reshape(-1) for p in ps])
    tp.comm.all_reduce(flat)
    off = 0
    for p in ps:
        n = p.numel()
        p.main_grad.copy_(flat[off:off + n].view(p.shape))
        off += n


def replicated_sqnorm(model: torch.nn.Module) -> torch.Tensor | None:
    ps = [p for p in replicated_params(model) if getattr(p, "main_grad", None) is not None]
    if not ps:
        return None
    return sum(p.main_grad.float().pow(2).sum() for p in ps)


# ----------------------------------------------------------------------------- sharding


def _gdn_qkv_rows(cfg: Any) -> list[int]:
    kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    return [kd, kd, cfg.linear_num_value_heads * cfg.linear_value_head_dim]


def shard_param(name: str, full: torch.Tensor, tp_rank: int, tp_size: int, cfg: Any) -> torch.Tensor:
    """The TP shard of a full (TP=1) parameter of a Qwen3Model, by parameter name."""
    if tp_size == 1:
        return full
    if name.endswith(("in_proj_qkv", "conv_weight")):  # Gated DeltaNet: [q; k; v] channels split by heads
        return torch.cat([t.chunk(tp_size, 0)[tp_rank] for t in full.split(_gdn_qkv_rows(cfg), 0)], 0)
    if name.endswith(("in_proj_z", "in_proj_b", "in_proj_a", "dt_bias", "A_log")):
        return full.chunk(tp_size, 0)[tp_rank]
    if name.endswith("out_proj"):
        return full.chunk(tp_size, 1)[tp_rank]
    if full.dim() < 2:
        return full
    d = cfg.head_dim
    if name.endswith("qkv_proj"):
        nq, nkv = cfg.num_attention_heads * d, cfg.num_key_value_heads * d
        q, k, v = full[:nq], full[nq:nq + nkv], full[nq + nkv:]
        pick = lambda t: t.chunk(tp_size, 0)[tp_rank]  # noqa: E731
        return torch.cat([pick(q), pick(k), pick(v)], 0)
    if name.endswith("gate_up_proj"):
        f = full.shape[0] // 2
        return torch.cat([full[:f].chunk(tp_size, 0)[tp_rank], full[f:].chunk(tp_size, 0)[tp_rank]], 0)
    if name.endswith(("o_proj", "down_proj")):
        return full.chunk(tp_size, 1)[tp_rank]
    if name.endswith(("embed_tokens", "lm_head", "attn_gate")):
        return full.chunk(tp_size, 0)[tp_rank]
    return full  # MoE experts / router: replicated over TP


def unshard_param(name: str, shards: list[torch.Tensor], cfg: Any) -> torch.Tensor:
    """Inverse of :func:`shard_param` given every rank's shard in rank order."""
    tp = len(shards)
    if tp == 1:
        return shards[0]
    if name.endswith(("in_proj_qkv", "conv_weight")):
        rows = [r // tp for r in _gdn_qkv_rows(cfg)]
        parts = [s.split(rows, 0) for s in shards]
        return torch.cat([torch.cat([p[i] for p in parts], 0) for i in range(3)], 0)
    if name.endswith(("in_proj_z", "in_proj_b", "in_proj_a", "dt_bias", "A_log")):
        return torch.cat(shards, 0)
    if name.endswith("out_proj"):
        return torch.cat(shards, 1)
    if shards[0].dim() < 2:
        return shards[0]
    d = cfg.head_dim
    if name.endswith("qkv_proj"):
        nq, nkv = cfg.num_attention_heads * d // tp, cfg.num_key_value_heads * d // tp
        q = torch.cat([s[:nq] for s in shards], 0)
        k = torch.cat([s[nq:nq + nkv] for s in shards], 0)
        v = torch.cat([s[nq + nkv:] for s in shards], 0)
        return torch.cat([q, k, v], 0)
    if name.endswith("gate_up_proj"):
        f = shards[0].shape[0] // 2
        return torch.cat([torch.cat([s[:f] for s in shards], 0), torch.cat([s[f:] for s in shards], 0)], 0)
    if name.endswith(("o_proj", "down_proj")):
        return torch.cat(shards, 1)
    if name.endswith(("embed_tokens", "lm_head", "attn_gate")):
        return torch.cat(shards, 0)
    return shards[0]


@torch.no_grad()
def load_shards_from_full(model: torch.nn.Module, full_state: dict[str, torch.Tensor], tp: TPContext) -> None:
    """Fill a TP-sharded model from a full (TP=1) ``named_parameters`` state."""
    for name, p in model.named_parameters():
        p.copy_(shard_param(name, full_state[name], tp.rank, tp.size, model.cfg).to(p.device, p.dtype))


@torch.no_grad()
def gather_full_state(model: torch.nn.Module, tp: TPContext) -> dict[str, torch.Tensor]:
    """Every parameter in its full (TP=1) shape, on every TP rank."""
    out = {}
    for name, p in model.named_parameters():
        if not tp.enabled or getattr(p, "tp_replicated", False):
            out[name] = p.detach().clone()
            continue
        x = p.detach().contiguous()
        parts = tp.comm.all_gather_rows(x[None]).view(tp.size, *x.shape)
        out[name] = unshard_param(name, list(parts.unbind(0)), model.cfg)
    return out
