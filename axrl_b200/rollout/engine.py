"""From-scratch rollout engine: paged KV cache, continuous batching, CUDA-graph decode bursts.

Reference counterpart: the SGLang engine driven by ``SGLangWorker``
(``axrl/worker/sglang_worker.py:49-851``): token-in/token-out generation with
sampled-token logprobs (:489-580), abort-and-continue for partial rollout
(:338-405, :710-726), routed-expert capture for R3 (:558-569), weight updates
(:761-796) and memory release/resume (:816-830).

Design (B200-first):
* KV lives in one tensor ``[L, 2, pages, Hkv, page_size, 128]`` bf16; the C++
  ``BlockManager`` owns page allocation, refcounts and the prefix cache;
* requests that share a prompt (a GRPO group) are prefilled ONCE; members share
  the prompt's full pages by refcount and copy the partial last page;
* prefill runs the packed range-list attention over new prompts while the fused
  q/k-norm+RoPE kernel scatters K/V into pages;
* decode is device-resident: one CUDA graph = one decode step (36 layers with
  residual adds fused into the GEMM epilogues, LM head, Gumbel-max sampler, and a
  bookkeeping kernel that feeds the sampled token back, advances positions and KV
  slots, forces EOS at prescribed lengths and appends to a token ring).  The host
  replays ``burst`` steps back to back and synchronises once per burst to collect
  tokens, retire finished rows and admit new requests.
"""

from __future__ import annotations

import dataclasses
import json
import math
import os
import time
import zlib
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch

from axrl_b200.models.qwen3 import Qwen3Model
from axrl_b200.ops import _ext
from axrl_b200.ops import core as ops
from axrl_b200.ops import paged
from axrl_b200.ops.attention_spec import spec_from_triples
from axrl_b200.rollout.kv import make_block_manager
from axrl_b200.utils import iostats


@dataclass
class GenRequest:
    rid: str
    prompt: list[int]
    max_new_tokens: int = 256
    temperature: float = 1.0
    stop_token_ids: tuple[int, ...] = ()
    forced_len: int | None = None  # end the response with `forced_token` at exactly this length
    forced_token: int | None = None
    capture_routing: bool = False
    seed_stream: int | None = None  # random stream id (defaults to a hash of rid)
    # sampling controls (defaults = plain temperature sampling on the fused kernel)
    top_k: int = -1
    top_p: float = 1.0
    min_p: float = 0.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    logit_bias: dict[int, float] | None = None
    allowed_token_ids: Sequence[int] | None = None  # constrained decoding: only these tokens may be drawn
    regex: str | None = None  # constrained decoding: the response must match this expression
    json_schema: Any = None  # ... or be JSON text of this schema (rollout/grammar.py subset)
    structural_tag: dict | None = None  # ... or free text whose tagged segments follow schemas
    gen_prefix: tuple[int, ...] = ()  # tokens generated before this request resumed (preemption)

    @property
    def constrained(self) -> bool:
        return self.regex is not None or self.json_schema is not None or self.structural_tag is not None

    @property
    def filtered(self) -> bool:
        return (self.top_k > 0 or self.top_p < 1.0 or self.min_p > 0.0 or self.presence_penalty != 0.0 or self.frequency_penalty != 0.0
                or self.repetition_penalty != 1.0 or bool(self.logit_bias) or self.allowed_token_ids is not None or self.constrained)


@dataclass
class GenResult:
    rid: str
    output_ids: list[int]
    output_logprobs: list[float]
    finish_reason: str  # "stop" | "length" | "abort"
    prompt_len: int
    cached_tokens: int = 0
    routed_experts: np.ndarray | None = None  # (prompt_len + n_out - 1, L, K) int16


@dataclass
class _Seq:
    req: GenRequest
    tokens: list[int]
    pages: list[int]
    out_ids: list[int] = field(default_factory=list)
    out_lps: list[float] = field(default_factory=list)
    stream: int = 0
    cached: int = 0
    routing: list = field(default_factory=list)
    end_total: int = 0  # total length at which the sequence ends
    force_eos: bool = False
    stop_on_eos: bool = False
    grammar: Any = None  # TokenGrammar of a constrained request
    gstate: int = 0  # its automaton state after the tokens generated so far
    lslot: int = -1  # slot of its linear-attention (Gated DeltaNet) states, hybrid models


def _stream_id(rid: str) -> int:
    return zlib.crc32(rid.encode()) & 0x7FFFFFFF


class RolloutEngine:
    def __init__(self, model: Qwen3Model, *, max_batch: int = 256, kv_tokens: int = 1 << 16, page_size: int = 64,
                 max_context: int = 16384, max_prefill_tokens: int = 16384, use_cuda_graph: bool = True, seed: int = 0,
                 eos_token_id: int | None = None, burst: int = 16, kv_memory_saver: bool = False, weight_format: str = "bf16",
                 tp_group: Any = None, embed_full: torch.Tensor | None = None, tokenizer: Any = None,
                 dp_attention: bool = False) -> None:
        self.model = model
        # data-parallel attention over an expert-parallel model: every EP rank serves its own requests
        # (own KV cache, own batch) and the ranks step in lockstep so each MoE layer's dispatch /
        # combine meets the same layer on every rank (a rank without work runs empty forwards)
        self.dp_attention = dp_attention
        if dp_attention:
            ep = getattr(model, "ep", None)
            if ep is None or not getattr(ep, "active", False):
                raise ValueError("dp_attention needs an expert-parallel MoE model")
            use_cuda_graph = False
        # lockstep decisions go over a group of their own (gloo, host tensors): an engine thread may
        # reach them while this rank's main thread still runs training collectives on the model's groups
        self._lock_group = (torch.distributed.new_group(backend="gloo")
                            if dp_attention and torch.distributed.is_initialized() and torch.distributed.get_world_size() > 1 else None)
        self.tokenizer = tokenizer  # token strings for grammar-constrained requests
        self._grammars: dict[tuple, Any] = {}
        self._token_strings: list[str] | None = None
        assert weight_format in ("bf16", "fp8_block")
        self.weight_format = weight_format
        self.fp8: dict[int, object] = {}
        cfg = model.cfg
        self.cfg = cfg
        p0 = next(model.parameters())
        self.device, self.dtype = p0.device, p0.dtype
        self.is_cuda = self.device.type == "cuda"
        self.P = page_size
        self.max_batch = max_batch
        self.max_context = max_context
        self.max_prefill_tokens = max_prefill_tokens
        self.eos = 0 if eos_token_id is None else eos_token_id
        self.burst = burst
        attn0 = next(layer.self_attn for layer in model.layers if hasattr(layer.self_attn, "nkv"))  # a full-attention layer
        L, Hkv, D = cfg.num_hidden_layers, attn0.nkv, cfg.head_dim
        self.num_pages = max(2, math.ceil(kv_tokens / page_size)) + 1  # last page: scratch for frozen/padded rows
        self.scratch_page = self.num_pages - 1
        self.kv_buf = None
        if self.is_cuda and kv_memory_saver:
            # KV pages live in a VMM-tagged region: released while the trainer runs, re-mapped at the
            # same address before the next rollout (captured decode graphs stay valid).
            from axrl_b200.runtime.vmm import VmmBuffer

            self.kv_buf = VmmBuffer((L, 2, self.num_pages, Hkv, page_size, D), self.dtype, tag=f"kv_cache_{id(self)}")
            self.kv = self.kv_buf.tensor
        else:
            self.kv = torch.zeros((L, 2, self.num_pages, Hkv, page_size, D), dtype=self.dtype, device=self.device)
        self.preempted: dict[str, _Seq] = {}
        self.bm = make_block_manager(self.num_pages - 1, page_size)
        self.max_pages = math.ceil(max_context / page_size) + 1
        self.ws = paged.DecodeWorkspace(max_batch, attn0.nq, max_context + page_size, self.device) if self.is_cuda else None
        self.use_graph = use_cuda_graph and self.is_cuda and not cfg.is_moe
        self.graphs: dict[int, tuple] = {}
        self.seed = seed
        self.gen = torch.Generator(device="cpu").manual_seed(seed)
        self.waiting: list[GenRequest] = []
        self.running: list[_Seq] = []
        self.stats = {"prefill_tokens": 0, "decode_steps": 0, "decode_tokens": 0, "prefill_s": 0.0, "decode_s": 0.0, "bursts": 0}
        if tp_group is not None and cfg.is_hybrid:
            raise NotImplementedError("tensor-parallel engines for hybrid (Gated DeltaNet) models are not built")
        self._alloc_static()
        self.tp = None
        if tp_group is not None and torch.distributed.get_world_size(tp_group) > 1:
            # tensor-parallel serving: `model` holds this rank's shards (local heads / FFN columns /
            # vocabulary rows); `embed_full` is the whole embedding table
            from axrl_b200.rollout.tp import RolloutTP

            assert self.is_cuda and not cfg.is_moe, "TP rollout serves dense models on GPUs"
            assert embed_full is not None and embed_full.shape[0] == cfg.vocab_size, "TP rollout needs the full embedding table"
            self.embed_full = embed_full
            self.tp = RolloutTP(tp_group, cfg.hidden_size, model.lm_weight.shape[0], max(max_prefill_tokens, max_batch), max_batch, self.dtype)
        if weight_format == "fp8_block":
            self.quantize_weights()

    # ------------------------------------------------------------------ fp8 serving
    def _dense_linear_weights(self) -> list[tuple[str, torch.Tensor]]:
        out = []
        for name, p in self.model.named_parameters():
            if name.endswith(("qkv_proj", "o_proj", "gate_up_proj", "down_proj")) and p.dim() == 2:
                out.append((name, p))
        return out

    @torch.no_grad()
    def quantize_weights(self) -> None:
        """Block-quantise every dense projection (128x128 e4m3 blocks + fp32 scales); embedding,
        norms and the LM head stay bf16."""
        from axrl_b200.ops.fp8 import Fp8Weight

        self.fp8 = {id(p): Fp8Weight.from_dense(p.detach()) for _, p in self._dense_linear_weights()}

    def set_fp8_weights(self, weights: dict[str, tuple[torch.Tensor, torch.Tensor]]) -> None:
        """Use externally produced block-fp8 weights (e.g. buffers written by the weight-sync push)."""
        from axrl_b200.ops.fp8 import Fp8Weight

        params = dict(self.model.named_parameters())
        for name, (q, s) in weights.items():
            self.fp8[id(params[name])] = Fp8Weight(q, s)

    # ------------------------------------------------------------------ static buffers
    def _alloc_static(self) -> None:
        B, dev = self.max_batch, self.device
        z = lambda dt, *shape: torch.zeros(*shape, dtype=dt, device=dev)  # noqa: E731
        self.st = {
            "tok": z(torch.int64, B), "pos": z(torch.int32, B), "len": z(torch.int32, B), "slot": z(torch.int64, B),
            "bt": z(torch.int32, B, self.max_pages), "temp": z(torch.float32, B), "rid": z(torch.int32, B),
            "forced": torch.full((B,), -1, dtype=torch.int64, device=dev), "end_total": z(torch.int32, B),
            "force_eos": z(torch.int32, B), "stop_on_eos": z(torch.int32, B), "lslot": torch.full((B,), B, dtype=torch.int64, device=dev),
        }
        # hybrid models: per-sequence Gated DeltaNet states (conv window + recurrent state), one slot
        # per running sequence; slot B is scratch for padded rows
        self.gdn_index = {li: i for i, li in enumerate(li for li in range(self.cfg.num_hidden_layers) if self.cfg.layer_is_linear(li))}
        self.gdn_free = list(range(B - 1, -1, -1))
        # the fused state-update kernel is opt-in until it has been validated on a B200
        self.gdn_kernel = self.is_cuda and os.environ.get("AXRL_GDN_KERNEL", "1") == "1"
        if self.gdn_index:
            a = self.model.layers[next(iter(self.gdn_index))].self_attn
            n = len(self.gdn_index)
            self.gdn_conv = z(torch.float32, n, B + 1, a.kernel - 1, a.conv_dim)
            self.gdn_S = z(torch.float32, n, B + 1, a.nv, a.dk, a.dv)
        self.s_seed = z(torch.int64, 1)
        # filtered sampling (top-k/p, min-p, penalties, bias / allowed set): per-row controls
        self.st.update({"top_k": torch.full((B,), -1, dtype=torch.int64, device=dev), "top_p": torch.ones(B, device=dev),
                        "min_p": z(torch.float32, B), "pres": z(torch.float32, B), "freq": z(torch.float32, B),
                        "rep": torch.ones(B, device=dev), "ngen": z(torch.int64, B)})
        self.hist_cap = 1024  # generated tokens remembered for the penalties (most recent)
        self.hist = torch.full((B, self.hist_cap), -1, dtype=torch.int64, device=dev)
        self.h_hist = torch.full((B, self.hist_cap), -1, dtype=torch.int64).pin_memory() if self.is_cuda else torch.full((B, self.hist_cap), -1, dtype=torch.int64)
        self.bias: torch.Tensor | None = None  # (B, V) additive logit bias, allocated on first use
        self.filtered_mode = False
        self.s_out_tok = z(torch.int64, B)
        self.s_out_lp = z(torch.float32, B)
        self.ring_cap = max(self.burst, 1)
        self.ring_tok = torch.full((self.ring_cap, B), -1, dtype=torch.int64, device=dev)
        self.ring_lp = z(torch.float32, self.ring_cap, B)
        self.ring_step = z(torch.int32, 1)
        pin = self.is_cuda
        self.h = {k: (torch.zeros_like(v, device="cpu").pin_memory() if pin else torch.zeros_like(v, device="cpu")) for k, v in self.st.items()}

    # ------------------------------------------------------------------ model pieces (inference, no autograd)
    def _lin(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        fw = self.fp8.get(id(w)) if self.fp8 else None
        if fw is not None:
            from axrl_b200.ops.fp8 import fp8_linear

            y = fp8_linear(x, fw)
            return y if residual is None else y + residual
        if self.is_cuda:
            e = _ext.ext()
            return e.linear_fwd(x, w) if residual is None else e.linear_residual(x, w, residual)
        y = torch.nn.functional.linear(x, w)
        return y if residual is None else y + residual

    def _rms(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if self.is_cuda:
            return _ext.ext().rmsnorm_fwd(x, w, self.cfg.rms_norm_eps)[0]
        return ops._rms_ref(x, w, self.cfg.rms_norm_eps)

    def _mlp(self, layer, x: torch.Tensor, h: torch.Tensor, capture: dict | None, li: int) -> torch.Tensor:  # noqa: ANN001
        mlp = layer.mlp
        if hasattr(mlp, "router"):
            from axrl_b200.models.moe import MoEContext

            return h + mlp(x, MoEContext(capture=capture), li)
        return self._lin(ops.swiglu(self._lin(x, mlp.gate_up_proj)), mlp.down_proj, residual=h)

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        if self.tp is not None:
            return _ext.ext().embed_fwd(ids, self.embed_full)
        if self.is_cuda:
            return _ext.ext().embed_fwd(ids, self.model.embed_tokens)
        return torch.nn.functional.embedding(ids, self.model.embed_tokens)

    def _layers_tp(self, h, pos, slots, attend):  # noqa: ANN001, ANN202
        """TP forward: local-shard GEMMs, one fused all-reduce + residual + RMSNorm after each
        row-parallel projection.  Returns the final normed hidden state."""
        tp, e, eps = self.tp, _ext.ext(), self.cfg.rms_norm_eps
        inv = self.model.inv_freq
        rows = h.shape[0]
        layers = self.model.layers
        x = self._rms(h, layers[0].input_layernorm.weight)
        for li, layer in enumerate(layers):
            a = layer.self_attn
            qkv = self._lin(x, a.qkv_proj)
            q, k, v = paged.qk_norm_rope_cache(qkv, a.q_norm, a.k_norm, pos, inv, a.nq, a.nkv, a.eps, self.kv[li, 0], self.kv[li, 1], slots)
            o = a.gate_output(attend(li, q, k, v).reshape(rows, -1), x, self._lin)
            self._lin_into(o, a.o_proj, tp.partial_buffer(rows))
            h, x = tp.allreduce_rms(rows, h, layer.post_attention_layernorm.weight, eps)
            g = ops.swiglu(self._lin(x, layer.mlp.gate_up_proj))
            self._lin_into(g, layer.mlp.down_proj, tp.partial_buffer(rows))
            nxt = layers[li + 1].input_layernorm.weight if li + 1 < len(layers) else self.model.norm.weight
            h, x = tp.allreduce_rms(rows, h, nxt, eps, want_h=li + 1 < len(layers))
        _ = e
        return x

    def _lin_into(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        fw = self.fp8.get(id(w)) if self.fp8 else None
        if fw is not None:
            from axrl_b200.ops.fp8 import fp8_linear

            out.copy_(fp8_linear(x, fw))
            return
        _ext.ext().linear_fwd_into(x.contiguous(), w, out)

    def _fold_elementwise(self, rows: int) -> bool:
        """Decode-size forwards (<= 128 rows) fold the RMSNorms before the qkv and gate/up projections
        and the SwiGLU before the down projection into the weight-streaming GEMMs (``linear_rms_stream``,
        ``linear_swiglu_stream``): three fewer kernels per layer.  Opt-in: ``AXRL_DECODE_FOLD=1``."""
        return (self.is_cuda and not self.fp8 and 1 <= rows <= 128 and self.cfg.hidden_size % 64 == 0
                and os.environ.get("AXRL_DECODE_FOLD", "0") == "1")

    def _layers(self, h, pos, slots, attend, capture=None, mix=None):  # noqa: ANN001, ANN202
        """``mix(li, module, x)``: the token mixer of linear-attention layers (hybrid models)."""
        if self.tp is not None:
            return self._layers_tp(h, pos, slots, attend)
        inv = self.model.inv_freq
        fold = self._fold_elementwise(h.shape[0])
        e = _ext.ext() if fold else None
        eps = self.cfg.rms_norm_eps
        for li, layer in enumerate(self.model.layers):
            a = layer.self_attn
            if li in self.gdn_index:
                x = self._rms(h, layer.input_layernorm.weight)
                h = h + mix(li, a, x)
                x = self._rms(h, layer.post_attention_layernorm.weight)
                h = self._mlp(layer, x, h, capture, li)
                continue
            if fold and a.attn_gate is None:
                x = None
                qkv = e.linear_rms_stream(h, layer.input_layernorm.weight, eps, a.qkv_proj)
            else:
                x = self._rms(h, layer.input_layernorm.weight)
                qkv = self._lin(x, a.qkv_proj)
            q, k, v = paged.qk_norm_rope_cache(qkv, a.q_norm, a.k_norm, pos, inv, a.nq, a.nkv, a.eps,
                                               self.kv[li, 0], self.kv[li, 1], slots)
            o = a.gate_output(attend(li, q, k, v).reshape(q.shape[0], -1), x, self._lin)
            h = self._lin(o, a.o_proj, residual=h)
            if fold and not hasattr(layer.mlp, "router"):
                gu = e.linear_rms_stream(h, layer.post_attention_layernorm.weight, eps, layer.mlp.gate_up_proj)
                h = e.linear_swiglu_stream(gu, layer.mlp.down_proj, h)
                continue
            x = self._rms(h, layer.post_attention_layernorm.weight)
            h = self._mlp(layer, x, h, capture, li)
        return self._rms(h, self.model.norm.weight)

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        if self.tp is not None:  # vocabulary shard on this rank, rows all-gathered
            rows = h.shape[0]
            self._lin_into(h, self.model.lm_weight, self.tp.logits_buffer(rows))
            return self.tp.gather_logits(rows)
        return self._lin(h, self.model.lm_weight)

    # ------------------------------------------------------------------ public API
    def add_requests(self, reqs: Sequence[GenRequest]) -> None:
        self.waiting.extend(reqs)

    def generate(self, reqs: Sequence[GenRequest]) -> list[GenResult]:
        """Run ``reqs`` to completion (continuous batching); results in request order.  With
        ``dp_attention`` this is collective over the EP group: every rank calls it (with its own
        requests, possibly none) and all return once no rank has work left."""
        self.add_requests(reqs)
        done: dict[str, GenResult] = {}
        while self._any_work():
            for r in self.step():
                done[r.rid] = r
        return [done[r.rid] for r in reqs]

    # ------------------------------------------------------------------ data-parallel attention
    def _ep_max(self, vals: list[int]) -> list[int]:
        """Element-wise max of small integers over every rank the MoE layers exchange rows with.  The
        max runs over the whole world (a superset of the EP x ETP grid: ranks of other EP groups only
        run a few more empty forwards) on the engine's own gloo group."""
        if self._lock_group is None:
            return vals
        t = torch.tensor(vals, dtype=torch.int64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=self._lock_group)
        return t.tolist()

    def _any_work(self) -> bool:
        local = bool(self.waiting or self.running)
        return bool(self._ep_max([int(local)])[0]) if self.dp_attention else local

    def _empty_forward(self) -> None:
        """The expert-parallel collectives of one forward with no tokens (a rank without work keeps
        the MoE layers of the other ranks' forward company)."""
        H = self.cfg.hidden_size
        x = torch.zeros(0, H, dtype=self.model.embed_tokens.dtype if self.model.embed_tokens is not None else torch.bfloat16,
                        device=self.device)
        with torch.no_grad():
            for li, layer in enumerate(self.model.layers):
                if hasattr(layer.mlp, "router"):
                    from axrl_b200.models.moe import MoEContext

                    layer.mlp(x, MoEContext(), li)

    def _step_dp(self) -> list[GenResult]:
        groups = self._plan_admission()
        finished: list[GenResult] = []
        if self._ep_max([int(bool(groups))])[0]:
            if groups:
                finished += self._prefill(groups)
            else:
                self._empty_forward()
        k = self._burst_len() if self.running else 0
        k_max = self._ep_max([k])[0]
        if k:
            finished += self._decode_burst(k)
        for _ in range(k_max - k):
            self._empty_forward()
        return finished

    def abort_all(self) -> list[GenResult]:
        """Stop every request now (partial rollout): running ones return their partial output."""
        out = [self._finish(s, "abort") for s in self.running]
        out += [self._unwrap(GenResult(r.rid, [], [], "abort", len(r.prompt))) for r in self.waiting]
        self.running, self.waiting = [], []
        return out

    def step(self) -> list[GenResult]:
        if self.dp_attention:
            return self._step_dp()
        if not self.is_cuda:
            finished = self._admit()
            return finished + (self._decode_burst() if self.running else [])
        # weights are read-only while the engine steps: weight-streaming GEMMs may start loading
        # them before the preceding kernel ends (programmatic dependent launch)
        e = _ext.ext()
        e.set_weights_static(True)
        try:
            finished = self._admit()
            if self.running:
                finished += self._decode_burst()
        finally:
            e.set_weights_static(False)
        return finished

    # ------------------------------------------------------------------ admission + prefill
    def _pages_needed(self, n_tokens: int) -> int:
        return -(-n_tokens // self.P)

    def _admit(self) -> list[GenResult]:
        groups = self._plan_admission()
        return self._prefill(groups) if groups else []

    def _plan_admission(self) -> list[list[GenRequest]]:
        """Requests admitted this step, grouped by identical prompt (removed from ``waiting``)."""
        if not self.waiting or len(self.running) >= self.max_batch:
            return []
        budget_seqs = self.max_batch - len(self.running)
        groups: dict[tuple, list[GenRequest]] = {}
        order: list[tuple] = []
        taken = tokens = 0
        for r in self.waiting:
            if taken >= budget_seqs:
                break
            key = tuple(r.prompt)
            if key not in groups:
                if tokens + len(r.prompt) > self.max_prefill_tokens and order:
                    continue
                groups[key] = []
                order.append(key)
                tokens += len(r.prompt)
            groups[key].append(r)
            taken += 1
        headroom = self._pages_needed(self.burst + 1)

        def need(key: tuple) -> int:
            n = len(key)
            return n // self.P + len(groups[key]) * ((1 if n % self.P else 0) + headroom)

        total = sum(need(k) for k in order)
        # keep the pages that running sequences need for their next burst, plus a 1% watermark:
        # admitting into that space would only force a preemption (and a re-prefill) next burst
        reserve = sum(max(0, self._pages_needed(min(len(s.tokens) + self.burst, s.end_total)) - len(s.pages)) for s in self.running)
        reserve += max(1, self.num_pages // 100) if self.running else 0
        while order and total + reserve > self.bm.num_available():
            total -= need(order[-1])
            del groups[order.pop()]
        if not order:
            if not self.running:
                raise RuntimeError("KV cache too small for a single request")
            return []
        admitted = {id(r) for key in order for r in groups[key]}
        self.waiting = [r for r in self.waiting if id(r) not in admitted]
        return [groups[k] for k in order]

    def _prefill(self, groups: list[list[GenRequest]]) -> list[GenResult]:
        t0 = time.perf_counter()
        ids, pos, slots, triples, lasts = [], [], [], [], []
        protos: list[_Seq] = []
        off = 0
        for members in groups:
            r0 = members[0]
            n = len(r0.prompt)
            assert 0 < n < self.max_context, f"prompt length {n} out of range"
            pages = self.bm.allocate(self._pages_needed(n))
            protos.append(_Seq(r0, list(r0.prompt), pages))
            ids.extend(r0.prompt)
            pos.extend(range(n))
            pg = np.asarray(pages, dtype=np.int64)
            ar = np.arange(n)
            slots.extend((pg[ar // self.P] * self.P + ar % self.P).tolist())
            triples.append((off, off + n, off, off + n, 1))
            lasts.append(off + n - 1)
            off += n
        dev = self.device
        ids_t = torch.tensor(ids, dtype=torch.int64).to(dev, non_blocking=True)
        pos_t = torch.tensor(pos, dtype=torch.int32).to(dev, non_blocking=True)
        slots_t = torch.tensor(slots, dtype=torch.int64).to(dev, non_blocking=True)
        spec = spec_from_triples(triples, off)
        if self.is_cuda:
            spec = spec.to(dev)
            iostats.add_h2d(ids_t, pos_t, slots_t, spec.qseg, spec.kr, spec.kseg, spec.qr, spec.fwd_tiles, spec.bwd_tiles)
        capture = {} if self.cfg.is_moe and any(m.capture_routing for g in groups for m in g) else None
        lslots = [[self.gdn_free.pop() for _ in members] for members in groups] if self.gdn_index else None

        def gdn_prefill(li: int, a, x: torch.Tensor) -> torch.Tensor:  # noqa: ANN001
            states: list = []
            out = a.forward(x, None, None, spec, states=states)
            gi = self.gdn_index[li]
            for (cs, S), sl in zip(states, lslots):  # every member of a group starts from the prompt's state
                for slot in sl:
                    self.gdn_conv[gi, slot].copy_(cs)
                    self.gdn_S[gi, slot].copy_(S)
            return out

        with torch.no_grad():
            h = self._embed(ids_t)
            h = self._layers(h, pos_t, slots_t, lambda li, q, k, v: ops.attention(q, k, v, spec), capture, mix=gdn_prefill)
            logits = self._logits(h.index_select(0, torch.tensor(lasts, device=dev)))
        rows, temps, rids, forced = [], [], [], []
        new_seqs: list[_Seq] = []
        for gi, members in enumerate(groups):
            proto = protos[gi]
            n = len(proto.tokens)
            full = n // self.P
            self.bm.insert([int(t) for t in proto.tokens], proto.pages)
            for mi, r in enumerate(members):
                if mi == 0:
                    s = proto
                else:
                    shared = proto.pages[:full]
                    self.bm.incref(shared)
                    extra = self.bm.allocate(len(proto.pages) - full)
                    if extra:
                        self.kv[:, :, extra[0]].copy_(self.kv[:, :, proto.pages[full]])
                    s = _Seq(r, list(r.prompt), shared + extra)
                s.stream = r.seed_stream if r.seed_stream is not None else _stream_id(r.rid)
                if lslots is not None:
                    s.lslot = lslots[gi][mi]
                if r.constrained:
                    s.grammar = self._grammar(r)
                    s.gstate = s.grammar.start
                    for t in r.gen_prefix:
                        s.gstate = s.grammar.advance(s.gstate, t)
                s.end_total = min(n + (r.forced_len if r.forced_len is not None else r.max_new_tokens), self.max_context)
                s.force_eos = r.forced_len is not None
                s.stop_on_eos = (self.eos in r.stop_token_ids) and r.forced_len is None
                if capture is not None and r.capture_routing:
                    o0 = sum(len(g[0].prompt) for g in groups[:gi])
                    s.routing.append(np.stack([capture[li][o0:o0 + n - 1].cpu().numpy() for li in sorted(capture)], 1))
                new_seqs.append(s)
                rows.append(gi)
                temps.append(r.temperature)
                rids.append(s.stream)
                forced.append(self.eos if (s.force_eos and n + 1 == s.end_total) else -1)
        lg = logits.index_select(0, torch.tensor(rows, device=dev))
        if any(s.req.filtered for s in new_seqs):
            rq = [s.req for s in new_seqs]
            as_t = lambda vals, dt: torch.tensor(vals, dtype=dt).to(dev)  # noqa: E731
            b = self._bias_rows(new_seqs, len(rq))
            tok, lp = paged.sample_filtered(lg, as_t(temps, torch.float32), as_t([r.top_k for r in rq], torch.int64),
                                            as_t([r.top_p for r in rq], torch.float32), as_t([r.min_p for r in rq], torch.float32),
                                            bias=None if b is None else b.to(dev), forced=as_t(forced, torch.int64),
                                            generator=None if self.is_cuda else self.gen)
        else:
            tok, lp = self._sample_rows(lg, temps, rids, forced)
        self.stats["prefill_tokens"] += off
        self.stats["prefill_s"] += time.perf_counter() - t0
        finished = []
        for s, t, l in zip(new_seqs, tok.tolist(), lp.tolist()):
            if self._accept(s, t, l):
                finished.append(self._finish(s, self._reason(s)))
            else:
                self.running.append(s)
        return finished

    def _sample_rows(self, logits, temps, rids, forced):  # noqa: ANN001, ANN202
        dev = self.device
        t = torch.tensor(temps, dtype=torch.float32).to(dev)
        f = torch.tensor(forced, dtype=torch.int64).to(dev)
        if self.is_cuda:
            self.s_seed.add_(1)
            return paged.sample(logits, t, self.s_seed, row_ids=torch.tensor(rids, dtype=torch.int32).to(dev), forced=f)
        return paged.sample(logits, t, torch.zeros(1, dtype=torch.int64), generator=self.gen, forced=f)

    def _accept(self, s: _Seq, tok: int, lp: float) -> bool:
        """Append one sampled token; return True when the sequence is finished."""
        s.tokens.append(tok)
        s.out_ids.append(tok)
        s.out_lps.append(lp)
        if s.grammar is not None:
            s.gstate = s.grammar.advance(s.gstate, tok)
        return len(s.tokens) >= s.end_total or (s.stop_on_eos and tok == self.eos) or (tok in s.req.stop_token_ids and not s.force_eos)

    def _reason(self, s: _Seq) -> str:
        if s.force_eos and len(s.out_ids) >= (s.req.forced_len or 0):
            return "stop"
        if s.out_ids and s.out_ids[-1] in s.req.stop_token_ids and not s.force_eos:
            return "stop"
        return "length"

    def _free_lslot(self, s: _Seq) -> None:
        if s.lslot >= 0:
            self.gdn_free.append(s.lslot)
            s.lslot = -1

    def _finish(self, s: _Seq, reason: str) -> GenResult:
        self.bm.release(s.pages)
        self._free_lslot(s)
        routing = np.concatenate(s.routing, 0) if s.routing else None
        return self._unwrap(GenResult(s.req.rid, s.out_ids, s.out_lps, reason, len(s.req.prompt), s.cached, routing))

    def _unwrap(self, res: GenResult) -> GenResult:
        """Stitch a finished continuation of a preempted sequence onto what the sequence had produced
        before preemption (following the chain when it was preempted more than once).

        The continuation re-prefilled prompt + partial output, so its routing rows start at its
        first non-cached position and already cover the preempted part: keep the original rows and
        append the continuation's rows past them."""
        orig = self.preempted.pop(res.rid, None)
        if orig is None:
            return res
        routing = np.concatenate(orig.routing, 0) if orig.routing else None
        if res.routed_experts is not None:
            r0 = 0 if routing is None else routing.shape[0]
            tail = res.routed_experts[max(0, r0 - res.cached_tokens):]
            routing = tail if routing is None else np.concatenate([routing, tail], 0)
        return self._unwrap(GenResult(orig.req.rid, orig.out_ids + res.output_ids, orig.out_lps + res.output_logprobs, res.finish_reason,
                                      len(orig.req.prompt), orig.cached, routing))

    def _preempt(self, s: _Seq) -> None:
        """Free a running sequence's pages; it resumes later by re-prefilling prompt + partial output."""
        self.bm.release(s.pages)
        s.pages = []
        self._free_lslot(s)
        r = s.req
        done = len(s.out_ids)
        # same sampling controls; the tokens generated so far stay visible to penalties and grammars
        cont = dataclasses.replace(r, rid=f"{r.rid}~p{done}", prompt=list(s.tokens), max_new_tokens=max(1, r.max_new_tokens - done),
                                   forced_len=None if r.forced_len is None else r.forced_len - done, seed_stream=s.stream,
                                   gen_prefix=tuple(r.gen_prefix) + tuple(s.out_ids))
        self.preempted[cont.rid] = s
        self.waiting.insert(0, cont)
        self.stats["preempted"] = self.stats.get("preempted", 0) + 1

    def release_kv(self) -> None:
        """Give the KV memory back (colocated training phase).  Nothing may be running."""
        assert not self.running, "abort or finish generation before releasing the KV cache"
        self.bm.clear_cache()
        if self.kv_buf is not None:
            self.kv_buf.pause(backup=False)

    def acquire_kv(self) -> None:
        if self.kv_buf is not None:
            self.kv_buf.resume()

    # ------------------------------------------------------------------ decode bursts
    def _upload_state(self, B: int, bucket: int) -> None:
        h, P = self.h, self.P
        h["bt"][:bucket].zero_()
        for i, s in enumerate(self.running):
            n = len(s.tokens)
            h["tok"][i] = s.tokens[-1]
            h["pos"][i] = n - 1
            h["len"][i] = n
            h["slot"][i] = s.pages[(n - 1) // P] * P + (n - 1) % P
            h["bt"][i, : len(s.pages)] = torch.as_tensor(s.pages, dtype=torch.int32)
            h["temp"][i] = s.req.temperature
            h["rid"][i] = s.stream
            h["end_total"][i] = s.end_total
            h["force_eos"][i] = int(s.force_eos)
            h["stop_on_eos"][i] = int(s.stop_on_eos)
            h["forced"][i] = self.eos if (s.force_eos and n + 1 == s.end_total) else -1
            r = s.req
            h["top_k"][i], h["top_p"][i], h["min_p"][i] = r.top_k, r.top_p, r.min_p
            h["pres"][i], h["freq"][i], h["rep"][i] = r.presence_penalty, r.frequency_penalty, r.repetition_penalty
            h["ngen"][i] = min(len(s.out_ids), self.hist_cap - 1)
            h["lslot"][i] = s.lslot if s.lslot >= 0 else self.max_batch
        self.filtered_mode = any(s.req.filtered for s in self.running)
        if self.filtered_mode:
            self._upload_filters(self.running, bucket)
        if bucket > B:
            h["len"][B:bucket] = 0
            h["slot"][B:bucket] = self.scratch_page * P
            h["tok"][B:bucket] = 0
            h["pos"][B:bucket] = 0
            h["forced"][B:bucket] = -1
            h["end_total"][B:bucket] = 0
            h["lslot"][B:bucket] = self.max_batch
        for k, dst in self.st.items():
            dst[:bucket].copy_(h[k][:bucket], non_blocking=True)
            if self.is_cuda:
                iostats.add_h2d(h[k][:bucket])
        self.ring_step.zero_()

    def _bias_rows(self, seqs: list, n_rows: int) -> torch.Tensor | None:
        """(n_rows, V) additive bias from logit_bias / allowed_token_ids / the row's grammar state
        (None when unused)."""
        if not any(s.req.logit_bias or s.req.allowed_token_ids is not None or s.grammar is not None for s in seqs):
            return None
        V = self.cfg.vocab_size
        b = torch.zeros(n_rows, V, dtype=torch.float32)
        for i, s in enumerate(seqs):
            r = s.req
            if r.allowed_token_ids is not None:
                b[i].fill_(float("-inf"))
                b[i, torch.as_tensor(list(r.allowed_token_ids), dtype=torch.long)] = 0.0
            if s.grammar is not None:
                m = torch.from_numpy(s.grammar.allowed(s.gstate))
                b[i, :m.numel()].masked_fill_(~m, float("-inf"))
                b[i, m.numel():] = float("-inf")
            for t, v in (r.logit_bias or {}).items():
                b[i, int(t)] += float(v)
        return b

    def _grammar(self, r: GenRequest):  # noqa: ANN202
        """Token-level automaton of a constrained request (cached per expression / schema)."""
        from axrl_b200.rollout.grammar import StructuralTagGrammar, make_token_grammar

        enc = lambda x: json.dumps(x, sort_keys=True) if x is not None and not isinstance(x, str) else x  # noqa: E731
        key = (r.regex, enc(r.json_schema), enc(r.structural_tag), tuple(r.stop_token_ids))
        g = self._grammars.get(key)
        if g is None:
            if self._token_strings is None:
                if self.tokenizer is None:
                    raise ValueError("grammar-constrained requests need the engine's tokenizer")
                n = min(self.cfg.vocab_size, len(self.tokenizer)) if hasattr(self.tokenizer, "__len__") else self.cfg.vocab_size
                self._token_strings = [self.tokenizer.decode([i]) for i in range(n)]
            eos = [self.eos] if self.eos is not None else []
            eos_ids = eos + [t for t in r.stop_token_ids if t not in eos]
            if r.structural_tag is not None:
                tag = json.loads(r.structural_tag) if isinstance(r.structural_tag, str) else r.structural_tag
                g = StructuralTagGrammar(tag["structures"], tag["triggers"], self._token_strings, eos_ids)
            else:
                g = make_token_grammar(regex=r.regex, json_schema=r.json_schema, token_strings=self._token_strings, eos_ids=eos_ids)
            self._grammars[key] = g
        return g

    def _upload_filters(self, seqs: list, bucket: int) -> None:
        self.h_hist.fill_(-1)
        for i, s in enumerate(seqs):
            tail = (list(s.req.gen_prefix) + s.out_ids)[-(self.hist_cap - 1):]
            if tail:
                self.h_hist[i, :len(tail)] = torch.as_tensor(tail, dtype=torch.int64)
        self.hist[:bucket].copy_(self.h_hist[:bucket], non_blocking=True)
        b = self._bias_rows(seqs, bucket)
        if b is not None:
            if self.bias is None:
                self.bias = torch.zeros(self.max_batch, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
            self.bias[:bucket].copy_(b.to(self.device), non_blocking=True)
        elif self.bias is not None:
            self.bias[:bucket].zero_()

    def _burst_len(self) -> int:
        # steps this burst: no row needs more than its remaining tokens
        remaining = max(s.end_total - len(s.tokens) for s in self.running)
        k = max(1, min(self.burst, remaining))
        if any(s.grammar is not None for s in self.running):
            k = 1  # a grammar's allowed set depends on the previous token: one step per burst
        return k

    def _decode_burst(self, k: int | None = None) -> list[GenResult]:
        t0 = time.perf_counter()
        k = self._burst_len() if k is None else k
        # pages for every position this burst may write; preempt the newest sequences when short
        while True:
            short = sum(max(0, self._pages_needed(min(len(s.tokens) + k, s.end_total)) - len(s.pages)) for s in self.running)
            if short <= self.bm.num_available() or len(self.running) <= 1:
                break
            self._preempt(self.running.pop())
        for s in self.running:
            need = self._pages_needed(min(len(s.tokens) + k, s.end_total))
            if need > len(s.pages):
                if self.bm.num_available() < need - len(s.pages):
                    raise RuntimeError("KV cache too small for a single sequence (raise kv_tokens)")
                s.pages.extend(self.bm.allocate(need - len(s.pages)))
        B = len(self.running)
        bucket = self._bucket(B)
        self._upload_state(B, bucket)
        capture = {} if self.cfg.is_moe and any(s.req.capture_routing for s in self.running) else None
        captured_rows = []
        with torch.no_grad():
            for _ in range(k):
                if self.use_graph:
                    self._replay(bucket)
                else:
                    self._decode_body(bucket, capture)
                    if capture is not None:
                        captured_rows.append(np.stack([capture[li][:B].cpu().numpy() for li in sorted(capture)], 1))
        toks = self.ring_tok[:k, :B].cpu()
        lps = self.ring_lp[:k, :B].cpu()
        if self.is_cuda:
            iostats.add_d2h(self.ring_tok[:k, :B], self.ring_lp[:k, :B])
        toks_l, lps_l = toks.T.tolist(), lps.T.tolist()
        finished, keep = [], []
        for i, s in enumerate(self.running):
            done = False
            for j in range(k):
                t = toks_l[i][j]
                if t < 0:
                    break
                if capture is not None and s.req.capture_routing:
                    s.routing.append(captured_rows[j][i:i + 1])
                if self._accept(s, t, lps_l[i][j]):
                    done = True
                    break
            if done:
                finished.append(self._finish(s, self._reason(s)))
            else:
                keep.append(s)
        self.running = keep
        self.stats["decode_steps"] += k
        self.stats["decode_tokens"] += B * k
        self.stats["bursts"] += 1
        self.stats["decode_s"] += time.perf_counter() - t0
        return finished

    def _bucket(self, B: int) -> int:
        if not self.use_graph:
            return B
        b = 8
        while b < B:
            b *= 2
        return min(b, self.max_batch)

    def _advance(self, bucket: int) -> None:
        st = self.st
        if self.is_cuda:
            _ext.ext().decode_advance(bucket, self.s_out_tok, self.s_out_lp, st["tok"], st["pos"], st["len"], st["slot"], st["bt"], self.P,
                                      st["end_total"], st["force_eos"], st["stop_on_eos"], self.eos, st["forced"], self.ring_tok,
                                      self.ring_lp, self.ring_step, self.scratch_page * self.P, self.s_seed)
            return
        # CPU reference of decode_advance
        step = int(self.ring_step[0]) % self.ring_cap
        for b in range(bucket):
            l = int(st["len"][b])
            if l <= 0:
                self.ring_tok[step, b] = -1
                continue
            t = int(self.s_out_tok[b])
            self.ring_tok[step, b] = t
            self.ring_lp[step, b] = self.s_out_lp[b]
            n = l + 1
            if n >= int(st["end_total"][b]) or (int(st["stop_on_eos"][b]) and t == self.eos):
                st["len"][b] = 0
                st["slot"][b] = self.scratch_page * self.P
                st["forced"][b] = -1
                continue
            st["tok"][b] = t
            st["pos"][b] = n - 1
            st["len"][b] = n
            st["slot"][b] = int(st["bt"][b, (n - 1) // self.P]) * self.P + (n - 1) % self.P
            st["forced"][b] = self.eos if (int(st["force_eos"][b]) and n + 1 == int(st["end_total"][b])) else -1
        self.ring_step += 1
        self.s_seed += 1

    def _decode_body(self, bucket: int, capture=None) -> None:  # noqa: ANN001
        st = self.st
        tok, pos, bt, lens, slots = st["tok"][:bucket], st["pos"][:bucket], st["bt"][:bucket], st["len"][:bucket], st["slot"][:bucket]
        if self.ws is not None:
            self.ws.plan(lens)  # one work list for all layers of this step
        h = self._embed(tok)
        lsl = st["lslot"][:bucket]

        def gdn_decode(li: int, a, x: torch.Tensor) -> torch.Tensor:  # noqa: ANN001
            gi = self.gdn_index[li]
            if self.gdn_kernel:  # recurrent update in place in the pool (csrc/kernels/gdn.cu)
                return a.step_pool(x, self.gdn_conv[gi], self.gdn_S[gi], lsl)
            conv, S = self.gdn_conv[gi].index_select(0, lsl), self.gdn_S[gi].index_select(0, lsl)
            out = a.step(x, conv, S)
            self.gdn_conv[gi].index_copy_(0, lsl, conv)
            self.gdn_S[gi].index_copy_(0, lsl, S)
            return out

        h = self._layers(h, pos, slots, lambda li, q, k, v: paged.paged_decode_attention(q, self.kv[li, 0], self.kv[li, 1], bt, lens, self.ws, planned=True),
                         capture, mix=gdn_decode)
        logits = self._logits(h)
        if self.filtered_mode:
            t, l = paged.sample_filtered(logits, st["temp"][:bucket], st["top_k"][:bucket], st["top_p"][:bucket], st["min_p"][:bucket],
                                         st["pres"][:bucket], st["freq"][:bucket], st["rep"][:bucket], self.hist[:bucket],
                                         self.bias[:bucket] if self.bias is not None else None, forced=st["forced"][:bucket],
                                         generator=None if self.is_cuda else self.gen)
            ng = st["ngen"][:bucket]
            self.hist[:bucket].scatter_(1, ng[:, None], t[:, None])
            ng.add_(1).clamp_(max=self.hist_cap - 1)
        elif self.is_cuda:
            t, l = paged.sample(logits, st["temp"][:bucket], self.s_seed, row_ids=st["rid"][:bucket], forced=st["forced"][:bucket])
        else:
            t, l = paged.sample(logits, st["temp"][:bucket], self.s_seed, generator=self.gen, forced=st["forced"][:bucket])
        self.s_out_tok[:bucket].copy_(t)
        self.s_out_lp[:bucket].copy_(l)
        self._advance(bucket)

    def _replay(self, bucket: int) -> None:
        key = (bucket, self.filtered_mode, self.bias is not None)
        g = self.graphs.get(key)
        if g is None:
            saved = {k: v.clone() for k, v in self.st.items()}
            saved_ring = (self.ring_tok.clone(), self.ring_lp.clone(), self.ring_step.clone(), self.s_seed.clone())
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._decode_body(bucket)
            torch.cuda.current_stream().wait_stream(s)
            # warm-up advanced the state: restore before capturing
            for k, v in saved.items():
                self.st[k].copy_(v)
            self.ring_tok.copy_(saved_ring[0]), self.ring_lp.copy_(saved_ring[1]), self.ring_step.copy_(saved_ring[2])
            self.s_seed.copy_(saved_ring[3])
            graph = torch.cuda.CUDAGraph()
            was = _ext._COUNT["enabled"]
            before = _ext.count_launches(True)
            with torch.cuda.graph(graph):
                self._decode_body(bucket)
            captured = _ext.count_launches(was) - before
            _ext._COUNT["launches"] = before
            self.graphs[key] = (graph, captured)
            g = self.graphs[key]
            # capture does not execute: state is still the restored one; run the first step for real
        g[0].replay()
        _ext.add_launches(g[1])

    def release_graphs(self) -> None:
        self.graphs.clear()

    # ------------------------------------------------------------------ weights / memory
    @torch.no_grad()
    def update_weights_from_model(self, src: Qwen3Model) -> None:
        """In-process weight sync: copy every parameter of ``src`` (same layout)."""
        for (n1, p1), (n2, p2) in zip(self.model.named_parameters(), src.named_parameters()):
            assert n1 == n2 and p1.shape == p2.shape, f"layout mismatch {n1} vs {n2}"
            p1.copy_(p2, non_blocking=True)
        if self.weight_format == "fp8_block":
            self.quantize_weights()

    def reset_prefix_cache(self) -> None:
        """Weights changed: cached pages no longer match (the reference flushes its radix cache)."""
        self.bm.clear_cache()
