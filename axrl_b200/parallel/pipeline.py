"""Pipeline parallelism: contiguous layer stages and the 1F1B schedule over NCCL point-to-point.

Reference: ``pp_size`` / ``vpp_size`` (``axrl/configs.py:379-380``), Megatron's
``forward_backward_pipelining_without_interleaving`` driven from
``axrl/worker/megatron_worker.py:950-1031``; activations move with NCCL p2p (kept on NCCL, as in
the reference, overlapped by batching each send with the opposite-direction receive).

Every stage of a pipeline receives the same packed micro-batches (they are built from the same
batch on every rank), so a stage knows every activation's shape without exchanging it.  Stage 0
embeds token ids; the last stage applies the final norm, the LM head and the loss.

Schedule (one-forward-one-backward): stage ``s`` of ``P`` runs ``P - s - 1`` warm-up forwards, then
alternates forward / backward, then drains the remaining backwards.  Communication per step is a
single batched ``isend`` + ``irecv`` pair (send forward output + receive backward gradient, or the
reverse), which cannot deadlock between neighbours.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.distributed as dist


@dataclass
class PPContext:
    size: int = 1
    rank: int = 0
    group: Any = None
    ranks: list[int] | None = None  # global ranks of the stages, in stage order
    vpp: int = 1  # virtual (interleaved) stages per rank

    @property
    def enabled(self) -> bool:
        return self.size > 1

    @property
    def is_first(self) -> bool:
        return self.rank == 0

    @property
    def is_last(self) -> bool:
        return self.rank == self.size - 1

    @classmethod
    def from_group(cls, group: Any, vpp: int = 1) -> "PPContext":
        if group is None or dist.get_world_size(group) == 1:
            return cls()
        ranks = dist.get_process_group_ranks(group)
        return cls(size=len(ranks), rank=dist.get_rank(group), group=group, ranks=ranks, vpp=max(1, vpp))

    def virtual(self, v: int) -> "PPContext":
        """Layer-range view of virtual stage ``v`` of ``size * vpp`` (chunk ``v // size`` of rank ``v % size``)."""
        return PPContext(size=self.size * self.vpp, rank=v, group=self.group, ranks=self.ranks)

    def layer_range(self, num_layers: int) -> tuple[int, int]:
        """Layers of this stage: an even split, earlier stages taking the remainder."""
        base, extra = divmod(num_layers, self.size)
        lo = self.rank * base + min(self.rank, extra)
        return lo, lo + base + (1 if self.rank < extra else 0)

    @property
    def prev(self) -> int | None:
        return None if self.is_first else self.ranks[self.rank - 1]

    @property
    def next(self) -> int | None:
        return None if self.is_last else self.ranks[self.rank + 1]


def _exchange(pp: PPContext, send: list[tuple[torch.Tensor, int]], recv: list[tuple[torch.Tensor, int]]) -> None:
    ops = [dist.P2POp(dist.isend, t, peer, group=pp.group) for t, peer in send]
    ops += [dist.P2POp(dist.irecv, t, peer, group=pp.group) for t, peer in recv]
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def run_1f1b(pp: PPContext, num_mb: int, act_shape: Callable[[int], tuple], act_dtype: torch.dtype, device: torch.device,
             forward: Callable[[int, torch.Tensor | None], torch.Tensor], loss: Callable[[int, torch.Tensor], torch.Tensor]) -> None:
    """Run forward+backward of ``num_mb`` micro-batches through this stage.

    ``forward(i, inp)`` runs the stage on micro-batch ``i`` (``inp`` is None on the first stage);
    ``loss(i, out)`` (last stage) returns the scalar to back-propagate; ``act_shape(i)`` is the shape
    of the activation sent between stages for micro-batch ``i``."""
    warm = min(pp.size - pp.rank - 1, num_mb)
    inputs: list[torch.Tensor | None] = [None] * num_mb
    outputs: list[torch.Tensor | None] = [None] * num_mb

    def recv_act(i: int) -> torch.Tensor | None:
        if pp.is_first:
            return None
        t = torch.empty(act_shape(i), dtype=act_dtype, device=device)
        _exchange(pp, [], [(t, pp.prev)])
        return t

    def do_forward(i: int, inp: torch.Tensor | None) -> None:
        if inp is not None:
            inp.requires_grad_(True)
        out = forward(i, inp)
        inputs[i] = inp
        outputs[i] = loss(i, out) if pp.is_last else out

    def do_backward(i: int, grad: torch.Tensor | None) -> torch.Tensor | None:
        out = outputs[i]
        if pp.is_last:
            out.backward()
        else:
            out.backward(grad)
        g = inputs[i].grad if inputs[i] is not None else None
        inputs[i] = outputs[i] = None
        return g

    # warm-up forwards
    for i in range(warm):
        do_forward(i, recv_act(i))
        if not pp.is_last:
            _exchange(pp, [(outputs[i].detach(), pp.next)], [])
    # steady state
    steady = num_mb - warm
    inp = recv_act(warm) if steady > 0 else None
    for j in range(steady):
        i_f, i_b = warm + j, j
        do_forward(i_f, inp)
        grad = None
        if not pp.is_last:  # send this forward's output, receive the gradient of micro-batch i_b
            grad = torch.empty(act_shape(i_b), dtype=act_dtype, device=device)
            _exchange(pp, [(outputs[i_f].detach(), pp.next)], [(grad, pp.next)])
        g_in = do_backward(i_b, grad)
        nxt = None
        sends = [(g_in, pp.prev)] if not pp.is_first else []
        recvs = []
        if j + 1 < steady and not pp.is_first:
            nxt = torch.empty(act_shape(warm + j + 1), dtype=act_dtype, device=device)
            recvs = [(nxt, pp.prev)]
        _exchange(pp, sends, recvs)
        inp = nxt
    # cool-down backwards
    for i_b in range(steady, num_mb):
        grad = None
        if not pp.is_last:
            grad = torch.empty(act_shape(i_b), dtype=act_dtype, device=device)
            _exchange(pp, [], [(grad, pp.next)])
        g_in = do_backward(i_b, grad)
        if not pp.is_first:
            _exchange(pp, [(g_in, pp.prev)], [])


def run_forward_only(pp: PPContext, num_mb: int, act_shape: Callable[[int], tuple], act_dtype: torch.dtype, device: torch.device,
                     forward: Callable[[int, torch.Tensor | None], torch.Tensor], consume: Callable[[int, torch.Tensor], None]) -> None:
    """Forward every micro-batch through the pipeline; the last stage calls ``consume(i, out)``."""
    for i in range(num_mb):
        inp = None
        if not pp.is_first:
            inp = torch.empty(act_shape(i), dtype=act_dtype, device=device)
            _exchange(pp, [], [(inp, pp.prev)])
        out = forward(i, inp)
        if pp.is_last:
            consume(i, out)
        else:
            _exchange(pp, [(out.contiguous(), pp.next)], [])


# ----------------------------------------------------------------------------- interleaved (virtual) stages
#
# With ``V`` virtual stages per rank, rank ``r`` holds model chunks ``c = 0..V-1``; chunk ``c`` is
# virtual stage ``v = c * P + r`` of ``P * V`` (layers split evenly over virtual stages), so an
# activation walks the ranks ``V`` times.  Per-rank action order (reference: Megatron's
# interleaved schedule behind ``virtual_pipeline_model_parallel_size``): micro-batches in groups of
# ``P``; within a group every chunk in turn; ``(P - r - 1) * 2 + (V - 1) * P`` warm-up forwards,
# then one forward / one backward, then the remaining backwards (chunks in reverse order).
#
# Communication is planned, not negotiated: every rank simulates the whole pipeline (all ranks'
# action lists, an action runs once its input has arrived) in ticks.  A tick is one action per
# rank followed by one batched exchange of the activations / gradients that tick produced, so
# both ends of every message know the tick and the order of its operations by construction, and
# the plan itself proves the schedule free of deadlock.


def interleaved_order(P: int, V: int, rank: int, num_mb: int, forward_only: bool = False) -> list[tuple[str, int, int]]:
    """Action list of ``rank``: ("F" | "B", micro-batch, chunk)."""
    fwd: list[tuple[int, int]] = []
    for g0 in range(0, num_mb, P):
        grp = range(g0, min(num_mb, g0 + P))
        for c in range(V):
            fwd += [(m, c) for m in grp]
    if forward_only:
        return [("F", m, c) for m, c in fwd]
    bwd: list[tuple[int, int]] = []
    for g0 in range(0, num_mb, P):
        grp = range(g0, min(num_mb, g0 + P))
        for c in reversed(range(V)):
            bwd += [(m, c) for m in grp]
    total = num_mb * V
    warm = min(total, (P - rank - 1) * 2 + (V - 1) * P)
    acts = [("F", *fwd[k]) for k in range(warm)]
    for j in range(total - warm):
        acts.append(("F", *fwd[warm + j]))
        acts.append(("B", *bwd[j]))
    acts += [("B", *bwd[k]) for k in range(total - warm, total)]
    return acts


@dataclass
class TickPlan:
    actions: list[list[tuple[str, int, int] | None]]  # [tick][rank]
    messages: list[list[tuple[str, int, int, int, int]]]  # [tick] -> (kind, src, dst, mb, dst virtual stage)


def plan_interleaved(P: int, V: int, num_mb: int, forward_only: bool = False) -> TickPlan:
    orders = [interleaved_order(P, V, r, num_mb, forward_only) for r in range(P)]
    last_v = P * V - 1
    ptr = [0] * P
    have_act: set[tuple[int, int]] = set()   # (virtual stage, mb) whose input activation has arrived
    have_grad: set[tuple[int, int]] = set()  # (virtual stage, mb) whose output gradient has arrived
    actions, messages = [], []
    while any(ptr[r] < len(orders[r]) for r in range(P)):
        acts: list = [None] * P
        msgs = []
        for r in range(P):
            if ptr[r] == len(orders[r]):
                continue
            kind, mb, c = orders[r][ptr[r]]
            v = c * P + r
            ok = (v == 0 or (v, mb) in have_act) if kind == "F" else (v == last_v or (v, mb) in have_grad)
            if not ok:
                continue
            acts[r] = (kind, mb, c)
            ptr[r] += 1
            if kind == "F" and v < last_v:
                msgs.append(("A", r, (v + 1) % P, mb, v + 1))
            elif kind == "B" and v > 0:
                msgs.append(("G", r, (v - 1) % P, mb, v - 1))
        if all(a is None for a in acts):
            # a ragged last group (num_mb % P != 0) can leave too few warm-up forwards: let the first
            # rank with a runnable forward further down its list run it now (deterministic, so
            # every rank derives the same plan)
            moved = False
            for r in range(P):
                for j in range(ptr[r] + 1, len(orders[r])):
                    kind, mb, c = orders[r][j]
                    v = c * P + r
                    if kind == "F" and (v == 0 or (v, mb) in have_act):
                        orders[r].insert(ptr[r], orders[r].pop(j))
                        moved = True
                        break
                if moved:
                    break
            if not moved:
                raise RuntimeError(f"interleaved schedule stalls (P={P}, V={V}, micro-batches={num_mb})")
            continue
        for kind, _src, _dst, mb, vd in msgs:
            (have_act if kind == "A" else have_grad).add((vd, mb))
        actions.append(acts)
        messages.append(sorted(msgs))
    return TickPlan(actions, messages)


def run_interleaved_1f1b(pp: PPContext, V: int, num_mb: int, act_shape: Callable[[int], tuple], act_dtype: torch.dtype,
                         device: torch.device, forward: Callable[[int, int, torch.Tensor | None], torch.Tensor],
                         loss: Callable[[int, torch.Tensor], torch.Tensor] | None = None,
                         consume: Callable[[int, torch.Tensor], None] | None = None) -> None:
    """Forward+backward of ``num_mb`` micro-batches through this rank's ``V`` chunks.

    ``forward(i, c, inp)`` runs chunk ``c`` on micro-batch ``i`` (``inp`` None for virtual stage 0);
    ``loss(i, out)`` is applied after the last virtual stage.  With ``consume`` instead of ``loss``
    the pipeline runs forward only and hands each last-stage output to ``consume(i, out)``."""
    P, r = pp.size, pp.rank
    forward_only = loss is None
    plan = plan_interleaved(P, V, num_mb, forward_only)
    last_v = P * V - 1
    inputs: dict[tuple[int, int], torch.Tensor | None] = {}
    outputs: dict[tuple[int, int], torch.Tensor] = {}
    arrived_act: dict[tuple[int, int], torch.Tensor] = {}
    arrived_grad: dict[tuple[int, int], torch.Tensor] = {}
    produced: dict[tuple[str, int, int], torch.Tensor] = {}
    _ensure_comm(pp)
    for acts, msgs in zip(plan.actions, plan.messages):
        a = acts[r]
        if a is not None:
            kind, mb, c = a
            v = c * P + r
            if kind == "F":
                inp = arrived_act.pop((v, mb), None) if v > 0 else None
                if inp is not None and not forward_only:
                    inp.requires_grad_(True)
                out = forward(mb, c, inp)
                if forward_only:
                    if v == last_v:
                        consume(mb, out)
                    else:
                        produced[("A", mb, v + 1)] = out.detach().contiguous()
                else:
                    inputs[(v, mb)] = inp
                    if v == last_v:
                        outputs[(v, mb)] = loss(mb, out)
                    else:
                        outputs[(v, mb)] = out
                        produced[("A", mb, v + 1)] = out.detach()
            else:
                out = outputs.pop((v, mb))
                if v == last_v:
                    out.backward()
                else:
                    out.backward(arrived_grad.pop((v, mb)))
                inp = inputs.pop((v, mb))
                if v > 0:
                    produced[("G", mb, v - 1)] = inp.grad
        send, recv = [], []
        for kind, src, dst, mb, vd in msgs:
            peer = pp.ranks[dst] if src == r else pp.ranks[src]
            if src == r:
                send.append((produced.pop((kind, mb, vd)), peer))
            elif dst == r:
                t = torch.empty(act_shape(mb), dtype=act_dtype, device=device)
                (arrived_act if kind == "A" else arrived_grad)[(vd, mb)] = t
                recv.append((t, peer))
        _exchange(pp, send, recv)


def _ensure_comm(pp: PPContext) -> None:
    """A first point-to-point batch must involve every rank of the group (NCCL): open it with a barrier."""
    if not getattr(pp, "_comm_ready", False):
        dist.barrier(group=pp.group)
        pp._comm_ready = True


def sync_tied_embedding_grads(model: torch.nn.Module, pp: PPContext, embed_group: Any) -> None:
    """With tied embeddings under PP the first and last stage each hold a copy; sum their grads."""
    if not pp.enabled or not model.cfg.tie_word_embeddings or embed_group is None:
        return
    if model.embed_tokens is not None and getattr(model.embed_tokens, "main_grad", None) is not None:
        dist.all_reduce(model.embed_tokens.main_grad, group=embed_group)
