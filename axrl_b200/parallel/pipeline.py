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
    def from_group(cls, group: Any) -> "PPContext":
        if group is None or dist.get_world_size(group) == 1:
            return cls()
        ranks = dist.get_process_group_ranks(group)
        return cls(size=len(ranks), rank=dist.get_rank(group), group=group, ranks=ranks)

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


def sync_tied_embedding_grads(model: torch.nn.Module, pp: PPContext, embed_group: Any) -> None:
    """With tied embeddings under PP the first and last stage each hold a copy; sum their grads."""
    if not pp.enabled or not model.cfg.tie_word_embeddings or embed_group is None:
        return
    if model.embed_tokens is not None and getattr(model.embed_tokens, "main_grad", None) is not None:
        dist.all_reduce(model.embed_tokens.main_grad, group=embed_group)
