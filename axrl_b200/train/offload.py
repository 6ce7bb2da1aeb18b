"""Host-memory offload for training state.

* :class:`AdamState` — the fp32 optimizer state of a flat parameter range (master weights and
  both Adam moments).  With ``fraction > 0`` the LAST ``fraction`` of the range lives in pinned
  host memory and its AdamW update runs on the CPU; the head stays on the GPU and is updated by
  the fused kernel.  This is the counterpart of Megatron's hybrid-device optimizer behind
  ``optimizer_cpu_offload`` / ``optimizer_offload_fraction`` (reference config
  ``axrl/configs.py:322``): 12 bytes of device memory per offloaded parameter are freed at the
  price of one device->host gradient copy and one host->device parameter copy per step.
* :func:`offload_activations` — a saved-tensor hook context that moves the activations autograd
  saves inside it to pinned host memory and brings them back for the backward, the counterpart of
  Megatron's activation CPU offloading (``cpu_offloading``, ``cpu_offloading_num_layers``,
  ``cpu_offloading_double_buffering``; ``axrl/worker/megatron_worker.py:844-846``).  With double
  buffering the copies run on a side stream, so the next layer's forward overlaps the previous
  layer's offload, and the backward prefetches ahead of use.
"""

from __future__ import annotations

import contextlib
from typing import Iterator

import torch


def offload_fraction(opt) -> float:  # noqa: ANN001
    """Fraction of optimizer state kept on the host for an optimizer config (0 when off)."""
    if not getattr(opt, "optimizer_cpu_offload", False):
        return 0.0
    f = float(getattr(opt, "optimizer_offload_fraction", 0.0))
    if not 0.0 <= f <= 1.0:
        raise ValueError(f"optimizer_offload_fraction must be in [0, 1], got {f}")
    return f


class AdamState:
    """fp32 master / exp_avg / exp_avg_sq of ``n`` elements, the tail ``fraction`` on the host."""

    def __init__(self, master: torch.Tensor, fraction: float = 0.0) -> None:
        n = master.numel()
        self.n = n
        self.device = master.device
        k = int(round(n * fraction)) if fraction > 0 else 0
        self.split = n - k
        pin = master.device.type == "cuda"
        self.dev_master = master[: self.split].contiguous() if k else master
        self.dev_m = torch.zeros_like(self.dev_master)
        self.dev_v = torch.zeros_like(self.dev_master)
        if k:
            self.host_master = torch.empty(k, dtype=torch.float32, pin_memory=pin)
            self.host_master.copy_(master[self.split:])
            self.host_m = torch.zeros(k, dtype=torch.float32, pin_memory=pin)
            self.host_v = torch.zeros(k, dtype=torch.float32, pin_memory=pin)
            self.host_grad = torch.empty(k, dtype=torch.float32, pin_memory=pin)
        else:
            self.host_master = self.host_m = self.host_v = self.host_grad = None
        self._pin = pin
        self.host_out: torch.Tensor | None = None  # parameter-dtype staging of the host part
        self._staging: torch.Tensor | None = None

    @property
    def offloaded(self) -> int:
        return self.n - self.split

    # ---------------------------------------------------------------- full views (checkpoints)
    def _full(self, dev: torch.Tensor, host: torch.Tensor | None) -> torch.Tensor:
        return dev if host is None else torch.cat([dev.cpu(), host])

    def master_full(self) -> torch.Tensor:
        return self._full(self.dev_master, self.host_master)

    def m_full(self) -> torch.Tensor:
        return self._full(self.dev_m, self.host_m)

    def v_full(self) -> torch.Tensor:
        return self._full(self.dev_v, self.host_v)

    @torch.no_grad()
    def load(self, master: torch.Tensor, m: torch.Tensor | None = None, v: torch.Tensor | None = None) -> None:
        for dev, host, src in ((self.dev_master, self.host_master, master), (self.dev_m, self.host_m, m), (self.dev_v, self.host_v, v)):
            if src is None:
                continue
            src = src.reshape(-1)
            dev.copy_(src[: self.split])
            if host is not None:
                host.copy_(src[self.split:])

    # ---------------------------------------------------------------- update
    def _staging_buf(self, n: int) -> torch.Tensor:
        if self._staging is None or self._staging.numel() < n:
            self._staging = torch.empty(n, dtype=torch.float32, device=self.device)
        return self._staging[:n]

    def step_range_p2p(self, lo: int, n: int, grad: torch.Tensor, peer_ptrs: torch.Tensor, s0: int, decay_n: int, lr: float, opt,  # noqa: ANN001
                       step: int, sqnorm: torch.Tensor, grad_scale: float) -> bool:
        """AdamW over [lo, lo + n) fused with the store of the new bf16 values into every rank's
        parameter buffer at element ``s0`` (``peer_ptrs``: int64 device pointers).  False (nothing
        done) when part of the range lives on the host or the sizes do not allow the fused kernel."""
        if self.device.type != "cuda" or lo + n > self.split or n % 8 or s0 % 8:
            return False
        from axrl_b200.ops import _ext

        _ext.ext().adamw_p2p_step(self.dev_master[lo:lo + n], grad[:n], self.dev_m[lo:lo + n], self.dev_v[lo:lo + n], peer_ptrs, s0,
                                  max(0, min(decay_n, n)), lr, opt.adam_beta1, opt.adam_beta2, opt.adam_eps, opt.weight_decay, step,
                                  sqnorm, float(opt.clip_grad), float(grad_scale))
        return True

    def step_range(self, lo: int, n: int, grad: torch.Tensor, out_bf16: torch.Tensor | None, decay_n: int, lr: float, opt,  # noqa: ANN001
                   step: int, sqnorm: torch.Tensor, grad_scale: float, need_master: bool = False) -> torch.Tensor | None:
        """AdamW over elements [lo, lo + n) of the state with gradient ``grad`` (n device floats).

        ``out_bf16`` (n elements, or None) receives the updated parameters.  With ``need_master``
        the updated fp32 masters of the range are returned as a device tensor (a view of the device
        state, or a staging buffer when part of the range is on the host)."""
        from axrl_b200.ops import _ext

        hi = lo + n
        d_hi = min(hi, self.split)
        if lo < d_hi:  # head on the GPU (fused kernel) or on the CPU when training on the CPU
            a, b = lo, d_hi
            dn = max(0, min(decay_n, b - a))
            out = None if out_bf16 is None else out_bf16[: b - a]
            if self.device.type == "cuda":
                _ext.ext().adamw_step(self.dev_master[a:b], grad[: b - a], self.dev_m[a:b], self.dev_v[a:b], out, dn, lr, opt.adam_beta1,
                                      opt.adam_beta2, opt.adam_eps, opt.weight_decay, step, sqnorm, float(opt.clip_grad),
                                      float(grad_scale))
            else:
                cpu_adamw(self.dev_master[a:b], grad[: b - a], self.dev_m[a:b], self.dev_v[a:b], dn, lr, opt, step, sqnorm, grad_scale)
                if out is not None:
                    out.copy_(self.dev_master[a:b])
        h_lo = max(lo, self.split)
        if h_lo < hi:  # tail on the host
            a, b = h_lo - self.split, hi - self.split
            g = self.host_grad[a:b]
            g.copy_(grad[h_lo - lo:], non_blocking=True)
            if self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()
            dn = max(0, min(decay_n - (h_lo - lo), b - a))
            cpu_adamw(self.host_master[a:b], g, self.host_m[a:b], self.host_v[a:b], dn, lr, opt, step, sqnorm.cpu(), grad_scale)
            if out_bf16 is not None:
                if self.host_out is None or self.host_out.dtype != out_bf16.dtype:
                    self.host_out = torch.empty(self.n - self.split, dtype=out_bf16.dtype, pin_memory=self._pin)
                hb = self.host_out[a:b]
                hb.copy_(self.host_master[a:b])
                out_bf16[h_lo - lo:].copy_(hb, non_blocking=True)
        if not need_master:
            return None
        if hi <= self.split:
            return self.dev_master[lo:hi]
        st = self._staging_buf(n)
        if lo < self.split:
            st[: self.split - lo].copy_(self.dev_master[lo:self.split])
        st[max(lo, self.split) - lo:].copy_(self.host_master[max(lo, self.split) - self.split:hi - self.split], non_blocking=True)
        return st


def cpu_adamw(m: torch.Tensor, g: torch.Tensor, ma: torch.Tensor, va: torch.Tensor, dec: int, lr: float, o, step: int,  # noqa: ANN001
              sqnorm: torch.Tensor, grad_scale: float) -> None:
    """AdamW with global-norm clipping on host (or CPU-training) tensors, in place."""
    g = g.float() * grad_scale
    if o.clip_grad > 0:
        norm = sqnorm.float().sqrt() * grad_scale
        g = g * torch.clamp(o.clip_grad / (norm + 1e-6), max=1.0)
    b1, b2 = o.adam_beta1, o.adam_beta2
    ma.mul_(b1).add_(g, alpha=1 - b1)
    va.mul_(b2).addcmul_(g, g, value=1 - b2)
    upd = (ma / (1 - b1 ** step)) / ((va / (1 - b2 ** step)).sqrt() + o.adam_eps)
    if dec:
        upd[:dec] += o.weight_decay * m[:dec]
    m.add_(upd, alpha=-lr)


# ------------------------------------------------------------------------------------ activations
class _Offloader:
    def __init__(self, double_buffer: bool) -> None:
        self.side = torch.cuda.Stream() if (double_buffer and torch.cuda.is_available()) else None

    def pack(self, t: torch.Tensor):  # noqa: ANN201
        if t.device.type != "cuda" or t.numel() < 1024 or isinstance(t, torch.nn.Parameter):
            return t  # small tensors and parameters stay where they are
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        if self.side is None:
            host.copy_(t)
            return (t.device, host, None, None)
        ev = torch.cuda.Event()
        ev.record()
        self.side.wait_event(ev)
        with torch.cuda.stream(self.side):
            host.copy_(t, non_blocking=True)
            t.record_stream(self.side)  # the device copy stays alive until the side stream read it
            done = torch.cuda.Event()
            done.record()
        return (t.device, host, done, None)

    def unpack(self, packed):  # noqa: ANN001, ANN201
        if isinstance(packed, torch.Tensor):
            return packed
        dev, host, done, _ = packed
        if done is not None:
            done.synchronize()  # the offload copy finished before the host buffer is read
        return host.to(dev, non_blocking=True)


@contextlib.contextmanager
def offload_activations(enabled: bool, double_buffer: bool = False) -> Iterator[None]:
    """Autograd saves the activations of the ops run inside this context to pinned host memory."""
    if not enabled:
        yield
        return
    o = _Offloader(double_buffer)
    with torch.autograd.graph.saved_tensors_hooks(o.pack, o.unpack):
        yield
