"""Block-scaled fp8 (e4m3) linear layers for rollout serving.

Weights carry one fp32 dequantisation scale per 128x128 block (the format the trainer->rollout
weight sync writes); activations are quantised per token and 128-wide K group on the fly.  The GEMM
is ``csrc/kernels/gemm_fp8_block.cu`` (tcgen05 kind::f8f6f4 with blockwise scaling).  The CPU path
dequantises and multiplies in fp32 (the oracle).

Reference counterpart: SGLang's blockwise-fp8 serving of the MoE checkpoints
(``tests/moe/test_fp8_mismatch_results.py:22-23``) and ``per_block_cast_to_fp8``
(``axrl/utils/megatron/fp8_quantizer.py:19,68``).
"""

from __future__ import annotations

import torch

from axrl_b200.ops import _ext

E4M3_MAX = 448.0
BLOCK = 128


def quantize_weight_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(N, K) -> e4m3 (N, K) and fp32 scales (ceil(N/128), ceil(K/128)) with w ~ q * s per block."""
    N, K = w.shape
    nb, kb = -(-N // BLOCK), -(-K // BLOCK)
    wp = torch.zeros(nb * BLOCK, kb * BLOCK, dtype=torch.float32, device=w.device)
    wp[:N, :K] = w.float()
    blocks = wp.view(nb, BLOCK, kb, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / E4M3_MAX
    q = (blocks / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).view(nb * BLOCK, kb * BLOCK)[:N, :K]
    return q.to(torch.float8_e4m3fn).contiguous(), s.contiguous()


def dequantize_weight_blocks(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    N, K = q.shape
    return q.float() * s.repeat_interleave(BLOCK, 0)[:N].repeat_interleave(BLOCK, 1)[:, :K]


def quantize_rows_ref(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    M, K = x.shape
    g = x.float().view(M, K // BLOCK, BLOCK)
    s = g.abs().amax(-1).clamp_min(1e-12) / E4M3_MAX
    q = (g / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(M, K)
    return q, s


class Fp8Weight:
    """A frozen block-quantised weight (rollout only; no autograd)."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor) -> None:
        self.q, self.s = q, s

    @classmethod
    def from_dense(cls, w: torch.Tensor) -> "Fp8Weight":
        return cls(*quantize_weight_blocks(w))

    @property
    def shape(self) -> torch.Size:
        return self.q.shape


def fp8_linear(x: torch.Tensor, w: Fp8Weight) -> torch.Tensor:
    """``x @ dequant(w).T`` with x quantised per (token, 128-group); bf16 result."""
    if not x.is_cuda:
        q, s = quantize_rows_ref(x)
        xd = q.float() * s.repeat_interleave(BLOCK, 1)
        return (xd @ dequantize_weight_blocks(w.q, w.s).t()).to(x.dtype)
    e = _ext.ext()
    xq, xs = e.quant_fp8_rows(x.contiguous())
    return e.fp8_block_linear(xq, xs, w.q, w.s)
