"""Qwen3 dense and MoE decoder (trainer side), written over ``axrl_b200.ops``.

The reference builds these models through Megatron-Bridge/TransformerEngine
(``axrl/worker/megatron_worker.py:817-915``).  Here the model is a plain
PyTorch module over this package's kernels, operating on *packed* tokens
(``(T,)`` ids, ``(T,)`` positions, an :class:`AttnSpec`) so the same code runs
flat varlen batches, prefix trees and CP shards.

Layout choices (B200-first):
* Q/K/V share one fused weight ``qkv_proj`` ((nq + 2 nkv) * D, H) and gate/up
  share ``gate_up_proj`` (2F, H): one GEMM each, activations written once;
* q/k RMSNorm + RoPE run in one kernel on the QKV GEMM output;
* the LM head is never materialised for a whole micro-batch: the logprob op
  chunks tokens and fuses log-softmax/label gather/entropy;
* parameters are bf16; the optimizer owns fp32 master copies and attaches
  ``main_grad`` fp32 buffers that weight-gradient GEMMs accumulate into.

HF names are produced by :func:`hf_state_dict` / consumed by
:func:`load_hf_state_dict` (split/concat of the fused weights).

Tensor parallelism (``tp``, a :class:`~axrl_b200.parallel.tensor_parallel.TPContext`) follows
Megatron with sequence parallelism: the hidden stream between blocks holds this rank's T/tp
token rows, QKV / gate-up are column-parallel (all-gather in), O / down row-parallel
(reduce-scatter out), embedding and LM head are vocabulary-parallel.
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field

import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

from axrl_b200.ops import core as ops
from axrl_b200.ops.attention_spec import AttnSpec
from axrl_b200.parallel import tensor_parallel as tpl
from axrl_b200.parallel.tensor_parallel import TPContext

_NO_TP = TPContext()


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 40960
    # MoE (num_experts == 0 -> dense)
    num_experts: int = 0
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list[int] = field(default_factory=list)
    initializer_range: float = 0.02
    # hybrid linear / full attention (Qwen3-Next / Qwen3.5 style): per-layer "linear_attention"
    # (Gated DeltaNet, models/gdn.py) or "full_attention"; None = every layer full attention
    layer_types: list[str] | None = None
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    # Qwen3-Next / Qwen3.5 full-attention and MoE specifics
    attn_output_gate: bool = False  # o <- o * sigmoid(x W_gate) per head before o_proj
    partial_rotary_factor: float = 1.0  # RoPE on the first rotary_dim of each head, the rest passed through
    zero_centered_norm: bool = False  # checkpoints store RMSNorm weights as offsets from 1
    shared_expert_intermediate_size: int = 0  # sigmoid-gated shared expert beside the routed ones

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def layer_is_linear(self, i: int) -> bool:
        return self.layer_types is not None and self.layer_types[i] == "linear_attention"

    @property
    def is_hybrid(self) -> bool:
        return self.layer_types is not None and "linear_attention" in self.layer_types

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_is_moe(self, i: int) -> bool:
        return self.is_moe and i not in self.mlp_only_layers and (i + 1) % self.decoder_sparse_step == 0

    def num_params(self) -> int:
        H, D = self.hidden_size, self.head_dim
        nq = self.num_attention_heads * (2 if self.attn_output_gate else 1)
        attn = H * (nq + 2 * self.num_key_value_heads) * D + self.num_attention_heads * D * H + 2 * D
        kd = self.linear_num_key_heads * self.linear_key_head_dim
        vd = self.linear_num_value_heads * self.linear_value_head_dim
        nv = self.linear_num_value_heads
        gdn = H * (2 * kd + vd) + (2 * kd + vd) * self.linear_conv_kernel_dim + H * vd + 2 * H * nv + 2 * nv + self.linear_value_head_dim + vd * H
        shared = (3 * H * self.shared_expert_intermediate_size + H) if self.shared_expert_intermediate_size else 0
        total = 0
        for i in range(self.num_hidden_layers):
            per = (gdn if self.layer_is_linear(i) else attn) + 2 * H
            if self.layer_is_moe(i):
                total += per + H * self.num_experts + self.num_experts * 3 * H * self.moe_intermediate_size + shared
            else:
                total += per + 3 * H * self.intermediate_size
        total += self.vocab_size * H * (1 if self.tie_word_embeddings else 2) + H
        return total

    @staticmethod
    def from_hf_dict(d: dict) -> "Qwen3Config":
        """From an HF ``config.json`` dict: Qwen3 / Qwen3-MoE, and Qwen3-Next / Qwen3.5 (dense or MoE,
        text model; a multimodal config's ``text_config`` is used)."""
        if "text_config" in d and "hidden_size" not in d:
            d = {**d["text_config"], "model_type": d["text_config"].get("model_type", d.get("model_type", ""))}
        keys = Qwen3Config.__dataclass_fields__.keys()
        kw = {k: d[k] for k in keys if k in d}
        if "head_dim" not in d and "hidden_size" in d:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        rope = d.get("rope_parameters") or {}
        for k in ("rope_theta", "partial_rotary_factor"):
            if k in rope:
                kw[k] = rope[k]
        if str(d.get("model_type", "")).startswith(("qwen3_next", "qwen3_5")):
            kw.setdefault("attn_output_gate", True)
            kw.setdefault("zero_centered_norm", True)
            if "layer_types" not in d and "full_attention_interval" in d:
                n = d["full_attention_interval"]
                kw["layer_types"] = ["linear_attention" if (i + 1) % n else "full_attention" for i in range(d["num_hidden_layers"])]
        return Qwen3Config(**kw)


PRESETS: dict[str, Qwen3Config] = {
    # Qwen3-8B shape: 36 layers, hidden 4096, 32q/8kv, head 128, FFN 12288, vocab 151936.
    "qwen3-8b": Qwen3Config(),
    # Qwen3-30B-A3B shape: 48 layers, hidden 2048, 32q/4kv, 128 experts top-8, expert FFN 768.
    "qwen3-30b-a3b": Qwen3Config(hidden_size=2048, intermediate_size=6144, num_hidden_layers=48, num_attention_heads=32,
                                 num_key_value_heads=4, head_dim=128, num_experts=128, num_experts_per_tok=8,
                                 moe_intermediate_size=768),
    "qwen3-0.6b": Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
                              num_key_value_heads=8, head_dim=128, tie_word_embeddings=True),
    # Plumbing-check model: 2 layers, hidden 256, 4 heads, FFN 768, vocab 1024.
    "tiny": Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=768, num_hidden_layers=2, num_attention_heads=4,
                        num_key_value_heads=4, head_dim=64, rope_theta=10000.0, tie_word_embeddings=False),
    "tiny-moe": Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=768, num_hidden_layers=2, num_attention_heads=4,
                            num_key_value_heads=2, head_dim=64, rope_theta=10000.0, num_experts=8, num_experts_per_tok=2,
                            moe_intermediate_size=128),
    # Hybrid plumbing model: 4 layers, three Gated DeltaNet layers per full-attention layer.
    "tiny-gdn": Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=768, num_hidden_layers=4, num_attention_heads=4,
                            num_key_value_heads=2, head_dim=64, rope_theta=10000.0,
                            layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
                            linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32),
    # Qwen3.5-35B-A3B shape: 40 layers (3 Gated DeltaNet : 1 gated full attention), hidden 2048, 16q/2kv,
    # head 256 with RoPE on the first 64 dims, 256 experts top-8 (FFN 512) + a shared expert (FFN 512),
    # vocab 248320.
    "qwen3.5-35b-a3b": Qwen3Config(vocab_size=248320, hidden_size=2048, intermediate_size=512, num_hidden_layers=40,
                                   num_attention_heads=16, num_key_value_heads=2, head_dim=256, rope_theta=10000.0,
                                   max_position_embeddings=32768, num_experts=256, num_experts_per_tok=8,
                                   moe_intermediate_size=512, shared_expert_intermediate_size=512,
                                   layer_types=["linear_attention" if (i + 1) % 4 else "full_attention" for i in range(40)],
                                   linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
                                   linear_value_head_dim=128, attn_output_gate=True, partial_rotary_factor=0.25,
                                   zero_centered_norm=True),
    # Plumbing model of the same family: 4 layers (3 GDN : 1 gated attention), MoE 8 experts top-2 + shared expert.
    "tiny-qwen3.5": Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=128, num_hidden_layers=4, num_attention_heads=4,
                                num_key_value_heads=2, head_dim=64, rope_theta=10000.0, num_experts=8, num_experts_per_tok=2,
                                moe_intermediate_size=128, shared_expert_intermediate_size=128,
                                layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
                                linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                                attn_output_gate=True, partial_rotary_factor=0.25, zero_centered_norm=True),
}


def resolve_preset(name: str) -> Qwen3Config:
    key = name.split(":", 1)[1] if name.startswith("synthetic:") else name
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, cfg: Qwen3Config, tp_size: int = 1) -> None:
        super().__init__()
        assert cfg.num_attention_heads % tp_size == 0 and cfg.num_key_value_heads % tp_size == 0
        self.nq = cfg.num_attention_heads // tp_size
        self.nkv = cfg.num_key_value_heads // tp_size
        self.d = cfg.head_dim
        self.eps = cfg.rms_norm_eps
        H = cfg.hidden_size
        self.qkv_proj = nn.Parameter(torch.empty((self.nq + 2 * self.nkv) * self.d, H))
        self.o_proj = nn.Parameter(torch.empty(H, self.nq * self.d))
        self.q_norm = nn.Parameter(torch.ones(self.d))
        self.k_norm = nn.Parameter(torch.ones(self.d))
        # output gate (Qwen3-Next / 3.5): a per-head sigmoid gate on the attention output, projected
        # from the same input as q; kept as its own weight so the fused q/k/v layout is unchanged
        self.attn_gate = nn.Parameter(torch.empty(self.nq * self.d, H)) if cfg.attn_output_gate else None
        self.cp = None  # context-parallel group (set by the model)
        self.stash = ops.AttnStash()  # attention outputs kept for the recompute in backward

    def gate_output(self, o: torch.Tensor, x: torch.Tensor, linear=None) -> torch.Tensor:  # noqa: ANN001
        """``o`` (rows, nq*d) times sigmoid of the gate projection of ``x`` (identity without a gate)."""
        if self.attn_gate is None:
            return o
        g = (linear or ops.linear)(x, self.attn_gate)
        return o * torch.sigmoid(g.float()).to(o.dtype)

    def forward(self, x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, spec: AttnSpec, tp: TPContext = _NO_TP) -> torch.Tensor:
        qkv = tpl.column_parallel_linear(x, self.qkv_proj, tp)
        q, k, v = ops.qk_norm_rope(qkv, self.q_norm, self.k_norm, pos, inv_freq, self.nq, self.nkv, self.eps)
        stash = self.stash if (self.training and torch.is_grad_enabled()) else None
        if self.cp is not None and self.cp.enabled:  # keys/values of every context-parallel rank
            from axrl_b200.parallel import context_parallel as cpx

            if cpx.ring_attention_supported(spec, self.cp):
                o = cpx.ring_attention(q, k, v, spec, self.cp, stash=stash)
            else:
                o = ops.attention(q, cpx.gather_kv(k, self.cp), cpx.gather_kv(v, self.cp), spec, stash=stash)
        else:
            o = ops.attention(q, k, v, spec, stash=stash)
        o = o.reshape(o.shape[0], -1)
        if self.attn_gate is not None:
            o = o * torch.sigmoid(tpl.column_parallel_linear(x, self.attn_gate, tp).float()).to(o.dtype)
        return tpl.row_parallel_linear(o, self.o_proj, tp)


class MLP(nn.Module):
    def __init__(self, hidden: int, ffn: int) -> None:
        super().__init__()
        self.gate_up_proj = nn.Parameter(torch.empty(2 * ffn, hidden))
        self.down_proj = nn.Parameter(torch.empty(hidden, ffn))

    def forward(self, x: torch.Tensor, tp: TPContext = _NO_TP) -> torch.Tensor:
        return tpl.row_parallel_linear(ops.swiglu(tpl.column_parallel_linear(x, self.gate_up_proj, tp)), self.down_proj, tp)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: Qwen3Config, layer_idx: int, tp_size: int = 1, ep=None) -> None:  # noqa: ANN001
        super().__init__()
        self.layer_idx = layer_idx
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        if cfg.layer_is_linear(layer_idx):
            from axrl_b200.models.gdn import GatedDeltaNet

            self.self_attn: nn.Module = GatedDeltaNet(cfg, tp_size)
        else:
            self.self_attn = Attention(cfg, tp_size)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        if cfg.layer_is_moe(layer_idx):
            from axrl_b200.models.moe import MoEBlock

            self.mlp: nn.Module = MoEBlock(cfg, ep)
        else:
            self.mlp = MLP(cfg.hidden_size, cfg.intermediate_size // tp_size)

    # selective recompute: submodules whose activations are recomputed in backward instead of
    # stored (Megatron's recompute_modules); set by the model from its RecomputePolicy
    selective: frozenset = frozenset()

    def _sel(self, name: str, fn, *args):  # noqa: ANN001, ANN002, ANN202
        if name in self.selective and torch.is_grad_enabled():
            return checkpoint(fn, *args, use_reentrant=False)
        return fn(*args)

    def forward(self, h: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, spec: AttnSpec, moe_ctx=None,  # noqa: ANN001
                tp: TPContext = _NO_TP) -> torch.Tensor:
        h = h + self.self_attn(self._sel("layernorm", self.input_layernorm, h), pos, inv_freq, spec, tp)
        x = self._sel("layernorm", self.post_attention_layernorm, h)
        if hasattr(self.mlp, "router"):
            if moe_ctx is not None and tp.enabled:
                moe_ctx = moe_ctx.rows(tp.rank * x.shape[0], (tp.rank + 1) * x.shape[0])
            if moe_ctx is not None:
                return h + self._sel("moe", self.mlp, x, moe_ctx, self.layer_idx)
            return h + self._sel("moe", self.mlp, x)
        return h + self._sel("mlp", self.mlp, x, tp)


SELECTIVE_MODULES = ("core_attn", "layernorm", "mlp", "moe", "shared_experts")


@dataclass
class RecomputePolicy:
    """Activation recompute and host offload of the decoder stack (Megatron's recompute_* and
    cpu_offloading* settings; reference ``axrl/configs.py:409-415``).

    * ``granularity="full"``: a layer's activations are recomputed from its input in backward.
      ``method="uniform"`` checkpoints groups of ``num_layers`` consecutive layers (default 1);
      ``method="block"`` checkpoints the first ``num_layers`` layers of this stage and stores the
      rest.
    * ``granularity="selective"``: only the listed ``modules`` are recomputed.  ``core_attn`` needs
      no extra work here: the attention kernels keep only the output and the log-sum-exp and always
      recompute the scores in backward.  ``layernorm``, ``mlp``, ``moe`` and ``shared_experts``
      recompute the norms, the dense MLP, the MoE block and the shared expert.
    * ``offload_layers``: the activations saved by the first ``offload_layers`` layers (those not
      recomputed) go to pinned host memory, on a side stream with ``offload_double_buffer``.
    """

    granularity: str | None = None
    method: str | None = None
    num_layers: int | None = None
    modules: tuple[str, ...] = ("core_attn",)
    offload_layers: int = 0
    offload_double_buffer: bool = False

    @classmethod
    def from_worker_config(cls, cfg) -> "RecomputePolicy":  # noqa: ANN001
        mods = tuple(cfg.recompute_modules) if cfg.recompute_modules else ("core_attn",)
        bad = [m for m in mods if m not in SELECTIVE_MODULES]
        if bad:
            raise ValueError(f"recompute_modules {bad} are not supported (supported: {list(SELECTIVE_MODULES)})")
        if cfg.recompute_granularity == "full" and cfg.recompute_method is None and cfg.recompute_num_layers not in (None, 1):
            raise ValueError("recompute_num_layers needs recompute_method ('uniform' or 'block')")
        if cfg.recompute_num_layers is not None and cfg.recompute_num_layers < (0 if cfg.recompute_method == "block" else 1):
            raise ValueError(f"recompute_num_layers must be positive, got {cfg.recompute_num_layers}")
        if cfg.cpu_offloading and cfg.cpu_offloading_num_layers < 1:
            raise ValueError("cpu_offloading needs cpu_offloading_num_layers >= 1")
        return cls(cfg.recompute_granularity, cfg.recompute_method, cfg.recompute_num_layers, mods,
                   cfg.cpu_offloading_num_layers if cfg.cpu_offloading else 0, bool(cfg.cpu_offloading_double_buffering))

    def groups(self, n_layers: int) -> list[tuple[int, int, bool]]:
        """(start, end, checkpointed) ranges covering the stage's layers in order."""
        if self.granularity != "full":
            return [(i, i + 1, False) for i in range(n_layers)]
        if self.method == "block":
            k = n_layers if self.num_layers is None else min(self.num_layers, n_layers)
            return [(i, i + 1, i < k) for i in range(n_layers)]
        g = max(1, self.num_layers or 1)
        return [(i, min(i + g, n_layers), True) for i in range(0, n_layers, g)]


class _LayerDone:
    def __init__(self, fn, idx: int) -> None:  # noqa: ANN001
        self.fn, self.idx = fn, idx

    def __call__(self, g: torch.Tensor) -> None:
        self.fn(self.idx)


def _run_layers(layers, h, pos, inv, spec, moe_ctx, tp):  # noqa: ANN001, ANN201
    for layer in layers:
        h = layer(h, pos, inv, spec, moe_ctx, tp)
    return h


class Qwen3Model(nn.Module):
    """Decoder stack.  ``forward`` returns final hidden states (T, H); the LM head
    is applied by :meth:`logprobs` (fused, chunked) or :meth:`logits`."""

    def __init__(self, cfg: Qwen3Config, tp_size: int = 1, tp: TPContext | None = None, ep=None, pp=None, cp=None) -> None:  # noqa: ANN001
        super().__init__()
        self.cfg = cfg
        self.cp = cp
        self.tp = tp or _NO_TP
        self.ep = ep
        self.pp = pp
        tp_size = self.tp.size if tp is not None else tp_size
        assert cfg.vocab_size % tp_size == 0, "vocabulary must split evenly over TP ranks"
        V = cfg.vocab_size // tp_size
        # pipeline stage: a contiguous block of layers; embedding on the first stage, final norm and
        # LM head on the last (a tied LM head is a copy of the embedding kept on the last stage)
        lo, hi = (0, cfg.num_hidden_layers) if pp is None else pp.layer_range(cfg.num_hidden_layers)
        self.layer_offset = lo
        self.first = pp is None or pp.is_first
        self.last = pp is None or pp.is_last
        self.embed_tokens = nn.Parameter(torch.empty(V, cfg.hidden_size)) if (self.first or (self.last and cfg.tie_word_embeddings)) else None
        self.layers = nn.ModuleList(DecoderLayer(cfg, i, tp_size, ep) for i in range(lo, hi))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps) if self.last else None
        self.lm_head = None if (cfg.tie_word_embeddings or not self.last) else nn.Parameter(torch.empty(V, cfg.hidden_size))
        self.register_buffer("inv_freq", ops.rope_inv_freq(cfg.rotary_dim, cfg.rope_theta), persistent=False)
        self.policy = RecomputePolicy()
        self.grad_ready_hook = None  # set by an optimizer that reduces gradients during backward
        for layer in self.layers:
            layer.self_attn.cp = cp
        if tp_size > 1:
            for name, p in self.named_parameters():
                if (p.dim() < 2 and not name.endswith(("dt_bias", "A_log"))) or ".mlp.router" in name or ".mlp.experts" in name \
                        or ".mlp.shared_" in name:
                    tpl.mark_replicated(p)

    @property
    def lm_weight(self) -> torch.Tensor:
        return self.embed_tokens if self.lm_head is None else self.lm_head

    @torch.no_grad()
    def init_weights(self, seed: int = 0) -> None:
        """Random init from ``seed`` (normal(0, 0.02), out-projections scaled by 1/sqrt(2L)).

        Each tensor draws from its own generator seeded by (seed, parameter name), so a tensor's
        values do not depend on which other tensors exist; TP-sharded tensors add the TP rank to
        the seed, TP-replicated ones do not (they must agree across ranks)."""
        std = self.cfg.initializer_range
        out_std = std / math.sqrt(2 * self.cfg.num_hidden_layers)
        for name, p in self.named_parameters():
            if p.dim() == 1:
                p.fill_(1.0)
                continue
            s = out_std if name.endswith(("o_proj", "down_proj", "out_proj")) else std
            ps = seed * 1000003 + zlib.crc32(self.global_name(name).encode())
            if self.tp.enabled and not getattr(p, "tp_replicated", False):
                ps += 7919 * self.tp.rank
            if getattr(p, "expert_parallel", False):
                ps += 104729 * self.ep.rank + 15485863 * self.ep.etp_rank
            if p.is_cuda:
                cg = torch.Generator(device=p.device).manual_seed(ps)
                p.normal_(0.0, s, generator=cg)
            else:
                g = torch.Generator(device="cpu").manual_seed(ps)
                p.copy_(torch.randn(p.shape, generator=g) * s)

    def global_name(self, name: str) -> str:
        """Parameter name with the global layer index (pipeline stages hold a slice of the layers)."""
        if self.layer_offset and name.startswith("layers."):
            i, rest = name[len("layers."):].split(".", 1)
            return f"layers.{int(i) + self.layer_offset}.{rest}"
        return name

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        """Token rows of ``ids`` (T,) -> hidden (T, H), or this TP rank's (T/tp, H) slice."""
        if self.tp.enabled:
            return tpl.vocab_parallel_embedding(ids, self.embed_tokens, self.tp)
        return ops.embedding(ids, self.embed_tokens)

    def forward(self, ids: torch.Tensor, pos: torch.Tensor, spec: AttnSpec, moe_ctx=None,  # noqa: ANN001
                hidden: torch.Tensor | None = None) -> torch.Tensor:
        """Final hidden states: (T, H), or (T/tp, H) rows of this rank under TP (T % tp == 0).

        A pipeline stage other than the first takes the previous stage's output as ``hidden``; a
        stage other than the last returns its raw output (no final norm)."""
        h = self.embed(ids) if self.first else hidden
        inv = self.inv_freq
        tp = self.tp
        hook = self.grad_ready_hook if torch.is_grad_enabled() else None
        pol = self.policy
        grad = torch.is_grad_enabled()
        from axrl_b200.train.offload import offload_activations

        for a, b, ckpt in pol.groups(len(self.layers)):
            group = self.layers[a:b]
            if hook is not None and h.requires_grad:
                # fires once the gradient of the group's input exists, i.e. the backward of its
                # layers (weight gradients included) has been issued
                for layer in group:
                    h.register_hook(_LayerDone(hook, layer.layer_idx))
            if ckpt and grad:
                ops.AttnStash.pushing = True  # the replay in backward reuses this forward's attention
                try:
                    h = checkpoint(_run_layers, group, h, pos, inv, spec, moe_ctx, tp, use_reentrant=False)
                finally:
                    ops.AttnStash.pushing = False
            else:
                with offload_activations(grad and a < pol.offload_layers, pol.offload_double_buffer):
                    h = _run_layers(group, h, pos, inv, spec, moe_ctx, tp)
        return self.norm(h) if self.last else h

    @property
    def recompute(self) -> bool:
        """Full per-layer recompute (the common setting); see :attr:`policy` for the others."""
        return self.policy.granularity == "full"

    @recompute.setter
    def recompute(self, on: bool) -> None:
        self.set_policy(RecomputePolicy("full") if on else RecomputePolicy())

    def set_policy(self, policy: RecomputePolicy) -> None:
        self.policy = policy
        sel = frozenset(policy.modules) if policy.granularity == "selective" else frozenset()
        for layer in self.layers:
            layer.selective = sel
            if hasattr(layer.mlp, "shared_selective"):
                layer.mlp.shared_selective = "shared_experts" in sel

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        assert not self.tp.enabled, "full logits are a rollout-side (TP=1) operation"
        return torch.nn.functional.linear(hidden.float(), self.lm_weight.float())

    def argmax_tokens(self, hidden: torch.Tensor) -> torch.Tensor:
        """Most likely token per row (TP=1; SFT accuracy)."""
        from axrl_b200.ops.logprob import argmax_tokens

        assert not self.tp.enabled, "argmax over a sharded vocabulary is not supported"
        return argmax_tokens(hidden, self.lm_weight)

    def logprobs(self, hidden: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0, entropy: bool = False,  # noqa: ANN201
                 entropy_top_k: int = 0):
        """Per-token log p(label) (and entropy) for all T tokens; under TP ``hidden`` is the SP slice
        and ``labels`` the full (T,) labels, and every TP rank returns the full result."""
        if self.tp.enabled:
            return tpl.vocab_parallel_logprob(tpl.gather_from_sp(hidden, self.tp), self.lm_weight, labels, self.tp,
                                              temperature=temperature, compute_entropy=entropy)
        from axrl_b200.ops.logprob import fused_logprob

        return fused_logprob(hidden, self.lm_weight, labels, temperature=temperature, compute_entropy=entropy, entropy_top_k=entropy_top_k)


# ----------------------------------------------------------------------------- HF naming


def _hf_entries(model: Qwen3Model) -> tuple[dict[str, torch.Tensor], dict]:
    """HF name -> tensor (a view of a parameter where the layouts agree), and, for names whose HF
    tensor is computed (zero-centered norm offsets, the interleaved q / gate rows of a gated q_proj),
    a writer that stores an HF tensor back into the parameters."""
    cfg = model.cfg
    out: dict[str, torch.Tensor] = {}
    writers: dict = {}

    def norm(name: str, w: torch.Tensor) -> None:
        if cfg.zero_centered_norm:  # HF stores (weight - 1); the kernels use the weight itself
            out[name] = w.detach() - 1.0
            writers[name] = lambda src, w=w: w.copy_(src.to(w.dtype) + 1.0)
        else:
            out[name] = w

    out["model.embed_tokens.weight"] = model.embed_tokens
    norm("model.norm.weight", model.norm.weight)
    if model.lm_head is not None:
        out["lm_head.weight"] = model.lm_head
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a = layer.self_attn
        norm(p + "input_layernorm.weight", layer.input_layernorm.weight)
        norm(p + "post_attention_layernorm.weight", layer.post_attention_layernorm.weight)
        if cfg.layer_is_linear(i):  # HF Qwen3-Next / 3.5 "linear_attn" names
            q = p + "linear_attn."
            out |= {q + "in_proj_qkv.weight": a.in_proj_qkv, q + "in_proj_z.weight": a.in_proj_z, q + "in_proj_b.weight": a.in_proj_b,
                    q + "in_proj_a.weight": a.in_proj_a, q + "conv1d.weight": a.conv_weight.unsqueeze(1), q + "dt_bias": a.dt_bias,
                    q + "A_log": a.A_log, q + "norm.weight": a.norm_weight, q + "out_proj.weight": a.out_proj}
        else:
            q, k, v = a.qkv_proj.split([a.nq * a.d, a.nkv * a.d, a.nkv * a.d], 0)
            out |= {p + "self_attn.k_proj.weight": k, p + "self_attn.v_proj.weight": v, p + "self_attn.o_proj.weight": a.o_proj}
            if a.attn_gate is not None:  # HF q_proj rows: [q_h; gate_h] per head
                name = p + "self_attn.q_proj.weight"
                out[name] = torch.stack([q.detach().view(a.nq, a.d, -1), a.attn_gate.detach().view(a.nq, a.d, -1)], 1).reshape(2 * a.nq * a.d, -1)

                def write(src: torch.Tensor, q=q, g=a.attn_gate, nq=a.nq, d=a.d) -> None:
                    s2 = src.view(nq, 2, d, -1)
                    q.copy_(s2[:, 0].reshape(nq * d, -1).to(q.dtype))
                    g.copy_(s2[:, 1].reshape(nq * d, -1).to(g.dtype))

                writers[name] = write
            else:
                out[p + "self_attn.q_proj.weight"] = q
            norm(p + "self_attn.q_norm.weight", a.q_norm)
            norm(p + "self_attn.k_norm.weight", a.k_norm)
        if cfg.layer_is_moe(i):
            out |= layer.mlp.hf_tensors(p)
        else:
            g, u = layer.mlp.gate_up_proj.chunk(2, 0)
            out |= {p + "mlp.gate_proj.weight": g, p + "mlp.up_proj.weight": u, p + "mlp.down_proj.weight": layer.mlp.down_proj}
    return out, writers


def hf_state_dict(model: Qwen3Model) -> dict[str, torch.Tensor]:
    """Unfused HF-named tensors (views where possible)."""
    return _hf_entries(model)[0]


def _normalise_hf_names(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Accept a multimodal checkpoint's text tower (``model.language_model.*``) and fused 3-D expert
    tensors (``mlp.experts.gate_up_proj`` (E, 2F, H) / ``mlp.experts.down_proj`` (E, H, F))."""
    out: dict[str, torch.Tensor] = {}
    for k, v in sd.items():
        if k.startswith("model.language_model."):
            k = "model." + k[len("model.language_model."):]
        elif k.startswith(("model.visual.", "visual.", "mtp.")):
            continue
        if k.endswith("mlp.experts.gate_up_proj") and v.dim() == 3:
            base, F = k[: -len("gate_up_proj")], v.shape[1] // 2
            for e in range(v.shape[0]):
                out[f"{base}{e}.gate_proj.weight"], out[f"{base}{e}.up_proj.weight"] = v[e, :F], v[e, F:]
            continue
        if k.endswith("mlp.experts.down_proj") and v.dim() == 3:
            base = k[: -len("down_proj")]
            for e in range(v.shape[0]):
                out[f"{base}{e}.down_proj.weight"] = v[e]
            continue
        out[k] = v
    return out


@torch.no_grad()
def load_hf_state_dict(model: Qwen3Model, sd: dict[str, torch.Tensor], strict: bool = True) -> list[str]:
    """Copy HF tensors into the fused parameters; returns missing names."""
    targets, writers = _hf_entries(model)
    sd = _normalise_hf_names(sd)
    missing = []
    for name, dst in targets.items():
        src = sd.get(name)
        if src is None:
            if name == "lm_head.weight" and "model.embed_tokens.weight" in sd:
                src = sd["model.embed_tokens.weight"]
            else:
                missing.append(name)
                continue
        if name in writers:
            writers[name](src)
        else:
            dst.copy_(src.to(dst.dtype))
    if strict and missing:
        raise KeyError(f"missing HF tensors: {missing[:8]}{'...' if len(missing) > 8 else ''}")
    return missing


class VirtualPipelineModel(nn.Module):
    """This rank's ``V`` chunks of an interleaved pipeline: chunk ``c`` is virtual stage
    ``c * P + r`` of ``P * V`` (reference: Megatron virtual pipeline stages,
    ``vpp_size`` in ``axrl/configs.py:380``).  Exposes the parts of :class:`Qwen3Model` the trainer
    uses; ``forward(..., chunk=c)`` runs one chunk."""

    def __init__(self, cfg: Qwen3Config, pp, tp: TPContext | None = None, ep=None, cp=None) -> None:  # noqa: ANN001
        super().__init__()
        self.cfg = cfg
        self.pp = pp
        self.vpp = pp.vpp
        self.chunks = nn.ModuleList(Qwen3Model(cfg, tp=tp, ep=ep, pp=pp.virtual(c * pp.size + pp.rank), cp=cp) for c in range(pp.vpp))
        self.tp = self.chunks[0].tp

    # ---- the Qwen3Model surface
    @property
    def first(self) -> bool:
        return self.chunks[0].first

    @property
    def last(self) -> bool:
        return self.chunks[-1].last

    @property
    def layers(self) -> list:
        return [layer for ch in self.chunks for layer in ch.layers]

    @property
    def embed_tokens(self):  # noqa: ANN201
        return self.chunks[0].embed_tokens

    @property
    def norm(self):  # noqa: ANN201
        return self.chunks[-1].norm

    @property
    def lm_head(self):  # noqa: ANN201
        return self.chunks[-1].lm_head

    @property
    def lm_weight(self) -> torch.Tensor:
        return self.chunks[-1].lm_weight

    @property
    def inv_freq(self) -> torch.Tensor:
        return self.chunks[0].inv_freq

    @inv_freq.setter
    def inv_freq(self, t: torch.Tensor) -> None:
        for ch in self.chunks:
            ch.inv_freq = t

    @property
    def recompute(self) -> bool:
        return self.chunks[0].recompute

    @recompute.setter
    def recompute(self, on: bool) -> None:
        for ch in self.chunks:
            ch.recompute = on

    def set_policy(self, policy: RecomputePolicy) -> None:
        for ch in self.chunks:
            ch.set_policy(policy)

    @property
    def grad_ready_hook(self):  # noqa: ANN201
        return self.chunks[0].grad_ready_hook

    @grad_ready_hook.setter
    def grad_ready_hook(self, fn) -> None:  # noqa: ANN001
        for ch in self.chunks:
            ch.grad_ready_hook = fn

    def init_weights(self, seed: int = 0) -> None:
        for ch in self.chunks:
            ch.init_weights(seed)

    def global_name(self, name: str) -> str:
        c, rest = name[len("chunks."):].split(".", 1)
        return self.chunks[int(c)].global_name(rest)

    def forward(self, ids: torch.Tensor, pos: torch.Tensor, spec: AttnSpec, moe_ctx=None, hidden: torch.Tensor | None = None,  # noqa: ANN001
                chunk: int = 0) -> torch.Tensor:
        return self.chunks[chunk](ids, pos, spec, moe_ctx, hidden=hidden)

    def logprobs(self, *a, **kw):  # noqa: ANN002, ANN003, ANN201
        return self.chunks[-1].logprobs(*a, **kw)

    def argmax_tokens(self, *a, **kw):  # noqa: ANN002, ANN003, ANN201
        return self.chunks[-1].argmax_tokens(*a, **kw)

