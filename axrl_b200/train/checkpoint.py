"""Checkpoint I/O: HF safetensors and a Megatron-compatible distributed checkpoint.

Reference: ``MegatronWorker`` save/load through Megatron-Bridge (``axrl/worker/megatron_worker.py:321-374,
443-466,782-796``), ``BaseController.save_checkpoint`` / ``save_hf_checkpoint`` (rotation, retries;
``axrl/controller/base_controller.py:153-244``).

* HF format: ``model.safetensors.index.json`` + shards with HF parameter names
  (``model.layers.{i}.self_attn.q_proj.weight`` ...), ``config.json``.
* Distributed format (``torch_dist`` backend, the format Megatron-Core writes): an
  ``iter_XXXXXXX/`` directory written with ``torch.distributed.checkpoint`` (``.metadata`` +
  ``*.distcp``), ``metadata.json`` naming the backend, ``common.pt`` for non-tensor state,
  ``latest_checkpointed_iteration.txt`` in the parent.  Tensor keys follow Megatron-Core naming
  with transformer layers stacked along a leading layer axis
  (``decoder.layers.self_attention.linear_qkv.weight`` of shape ``[L, ...]``), and the fused QKV
  weight is stored in Megatron's per-query-group interleaved order ``[q_g, k_g, v_g]`` for each
  KV group g.  Optimizer state (fp32 master weights and Adam moments) is stored under
  ``optimizer.*`` keys in the same stacked layout.  Under data parallelism each rank writes only
  its own shard of the optimizer state (DCP handles the global layout).
"""

from __future__ import annotations

import json
import os
import shutil
import time
from pathlib import Path
from typing import Any

import torch

from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model, hf_state_dict, load_hf_state_dict

# ----------------------------------------------------------------------------- HF safetensors


def save_hf_checkpoint(model: Qwen3Model, path: str | os.PathLike, max_shard_bytes: int = 5 << 30, dtype: torch.dtype = torch.bfloat16) -> None:
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    sd = {k: v.detach().to("cpu", dtype).contiguous() for k, v in hf_state_dict(model).items()}
    shards, cur, size = [], {}, 0
    for k, v in sd.items():
        n = v.numel() * v.element_size()
        if cur and size + n > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v
        size += n
    if cur:
        shards.append(cur)
    index = {"metadata": {"total_size": sum(v.numel() * v.element_size() for v in sd.values())}, "weight_map": {}}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, str(path / name), metadata={"format": "pt"})
        for k in sh:
            index["weight_map"][k] = name
    (path / "model.safetensors.index.json").write_text(json.dumps(index, indent=2))
    cfg = model.cfg
    if cfg.is_hybrid:  # Qwen3.5 / 3.6 text model (HF keeps the RoPE fraction in rope_parameters)
        arch, mtype = ("Qwen3_5MoeForCausalLM", "qwen3_5_moe_text") if cfg.is_moe else ("Qwen3_5ForCausalLM", "qwen3_5_text")
    else:
        arch, mtype = ("Qwen3MoeForCausalLM", "qwen3_moe") if cfg.is_moe else ("Qwen3ForCausalLM", "qwen3")
    hf_cfg = {"architectures": [arch], "model_type": mtype, "torch_dtype": str(dtype).replace("torch.", ""),
              **{k: getattr(cfg, k) for k in cfg.__dataclass_fields__}}
    if cfg.is_hybrid:
        hf_cfg["rope_parameters"] = {"rope_type": "default", "rope_theta": cfg.rope_theta, "partial_rotary_factor": cfg.partial_rotary_factor}
    (path / "config.json").write_text(json.dumps(hf_cfg, indent=2))


def read_hf_state_dict(path: str | os.PathLike) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    path = Path(path)
    idx = path / "model.safetensors.index.json"
    files = sorted(set(json.loads(idx.read_text())["weight_map"].values())) if idx.exists() else [p.name for p in path.glob("*.safetensors")]
    sd: dict[str, torch.Tensor] = {}
    for f in files:
        sd.update(load_file(str(path / f)))
    return sd


def load_hf_checkpoint(model: Qwen3Model, path: str | os.PathLike, strict: bool = True) -> list[str]:
    return load_hf_state_dict(model, read_hf_state_dict(path), strict=strict)


def hf_config(path: str | os.PathLike) -> Qwen3Config:
    return Qwen3Config.from_hf_dict(json.loads((Path(path) / "config.json").read_text()))


# ----------------------------------------------------------------------------- Megatron-style dist checkpoint


def _qkv_to_mcore(w: torch.Tensor, nq: int, nkv: int, d: int) -> torch.Tensor:
    q, k, v = w.split([nq * d, nkv * d, nkv * d], 0)
    g = nq // nkv
    q = q.view(nkv, g * d, -1)
    return torch.cat([q, k.view(nkv, d, -1), v.view(nkv, d, -1)], 1).reshape(w.shape)


def _qkv_from_mcore(w: torch.Tensor, nq: int, nkv: int, d: int) -> torch.Tensor:
    g = nq // nkv
    x = w.view(nkv, (g + 2) * d, -1)
    q, k, v = x.split([g * d, d, d], 1)
    return torch.cat([q.reshape(nq * d, -1), k.reshape(nkv * d, -1), v.reshape(nkv * d, -1)], 0)


def _mcore_entries(model: Qwen3Model) -> list[tuple[str, int | None, torch.Tensor, Any]]:
    """(Megatron-Core name, layer index or None, tensor in that layout, writer) for every tensor.

    Entries of the same name over all layers are stacked on axis 0; a hybrid model keys its
    token-mixer tensors per layer (``decoder.layers.{i}.*``) since the mixers differ.  Zero-centered
    RMSNorms (Qwen3-Next / 3.5) are stored as offsets from 1, like Megatron's zero-centered gamma."""
    cfg = model.cfg
    ents: list[tuple[str, int | None, torch.Tensor, Any]] = []

    def plain(name: str, i: int | None, p: torch.Tensor) -> None:
        ents.append((name, i, p.detach(), lambda src, p=p: p.copy_(src.to(p.dtype))))

    def norm(name: str, i: int | None, p: torch.Tensor) -> None:
        if cfg.zero_centered_norm:
            ents.append((name, i, p.detach() - 1.0, lambda src, p=p: p.copy_(src.to(p.dtype) + 1.0)))
        else:
            plain(name, i, p)

    plain("embedding.word_embeddings.weight", None, model.embed_tokens)
    norm("decoder.final_layernorm.weight", None, model.norm.weight)
    if model.lm_head is not None:
        plain("output_layer.weight", None, model.lm_head)
    for i, layer in enumerate(model.layers):
        a = layer.self_attn
        norm("decoder.layers.self_attention.linear_qkv.layer_norm_weight", i, layer.input_layernorm.weight)
        m = f"decoder.layers.{i}." if cfg.is_hybrid else "decoder.layers."  # mixer tensors of a hybrid model: per layer
        if cfg.layer_is_linear(i):
            for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "conv_weight", "dt_bias", "A_log", "norm_weight", "out_proj"):
                plain(m + f"linear_attention.{n}", None, getattr(a, n))
        else:
            li = None if cfg.is_hybrid else i
            ents.append((m + "self_attention.linear_qkv.weight", li, _qkv_to_mcore(a.qkv_proj.detach(), a.nq, a.nkv, a.d),
                         lambda src, a=a: a.qkv_proj.copy_(_qkv_from_mcore(src, a.nq, a.nkv, a.d).to(a.qkv_proj.dtype))))
            plain(m + "self_attention.linear_proj.weight", li, a.o_proj)
            norm(m + "self_attention.q_layernorm.weight", li, a.q_norm)
            norm(m + "self_attention.k_layernorm.weight", li, a.k_norm)
            if a.attn_gate is not None:
                plain(m + "self_attention.linear_gate.weight", li, a.attn_gate)
        mlp = layer.mlp
        if hasattr(mlp, "router"):
            norm("decoder.layers.pre_mlp_layernorm.weight", i, layer.post_attention_layernorm.weight)
            plain("decoder.layers.mlp.router.weight", i, mlp.router)
            plain("decoder.layers.mlp.experts.linear_fc1.weight", i, mlp.experts_gate_up)
            plain("decoder.layers.mlp.experts.linear_fc2.weight", i, mlp.experts_down)
            if mlp.shared_gate_up is not None:
                plain("decoder.layers.mlp.shared_experts.linear_fc1.weight", i, mlp.shared_gate_up)
                plain("decoder.layers.mlp.shared_experts.linear_fc2.weight", i, mlp.shared_down)
                plain("decoder.layers.mlp.shared_experts.gate_weight", i, mlp.shared_gate)
        else:
            norm("decoder.layers.mlp.linear_fc1.layer_norm_weight", i, layer.post_attention_layernorm.weight)
            plain("decoder.layers.mlp.linear_fc1.weight", i, mlp.gate_up_proj)
            plain("decoder.layers.mlp.linear_fc2.weight", i, mlp.down_proj)
    return ents


def mcore_state_dict(model: Qwen3Model) -> dict[str, torch.Tensor]:
    """Megatron-Core names, transformer layers stacked on axis 0."""
    L = model.cfg.num_hidden_layers
    out: dict[str, torch.Tensor] = {}
    per: dict[str, list[torch.Tensor]] = {}
    for name, i, t, _ in _mcore_entries(model):
        if i is None:
            out[name] = t
        else:
            per.setdefault(name, []).append(t)
    for k, vs in per.items():
        assert len(vs) == L, f"{k}: heterogeneous layers are not stacked"
        out[k] = torch.stack(vs, 0)
    return out


@torch.no_grad()
def load_mcore_state_dict(model: Qwen3Model, sd: dict[str, torch.Tensor]) -> None:
    for name, i, _, write in _mcore_entries(model):
        write(sd[name] if i is None else sd[name][i])


def _iter_dir(root: Path, step: int) -> Path:
    return root / f"iter_{step:07d}"


def save_dist_checkpoint(root: str | os.PathLike, step: int, model: Qwen3Model, optim: Any = None, extra: dict | None = None,
                         most_recent_k: int | None = 2, retries: int = 5) -> Path:
    """Write ``root/iter_{step:07d}`` (torch_dist backend) and update the latest-iteration marker."""
    import torch.distributed.checkpoint as dcp

    root = Path(root)
    d = _iter_dir(root, step)
    state: dict[str, Any] = {f"model.{k}": v.to("cpu") for k, v in mcore_state_dict(model).items()}
    if optim is not None:
        for k, v in optim.state_dict().items():
            if isinstance(v, torch.Tensor):  # sharded optimizers name their slices per rank
                state[f"optimizer.{k}"] = v.detach().to("cpu")
    rank = torch.distributed.get_rank() if torch.distributed.is_initialized() else 0
    for attempt in range(retries):
        try:
            d.mkdir(parents=True, exist_ok=True)
            dcp.save(state, checkpoint_id=str(d))
            if rank == 0:
                (d / "metadata.json").write_text(json.dumps({"sharded_backend": "torch_dist", "sharded_backend_version": 1,
                                                             "common_backend": "torch", "common_backend_version": 1}))
                torch.save({"iteration": step, "optimizer_step": getattr(optim, "step_count", 0), "extra": extra or {}}, d / "common.pt")
                (root / "latest_checkpointed_iteration.txt").write_text(str(step))
            break
        except OSError:
            if attempt == retries - 1:
                raise
            time.sleep(2 ** attempt)
    if rank == 0 and most_recent_k:
        iters = sorted(p for p in root.glob("iter_*") if p.is_dir())
        for old in iters[:-most_recent_k]:
            shutil.rmtree(old, ignore_errors=True)
    return d


def latest_iteration(root: str | os.PathLike) -> int | None:
    f = Path(root) / "latest_checkpointed_iteration.txt"
    return int(f.read_text().strip()) if f.exists() else None


def load_dist_checkpoint(root: str | os.PathLike, model: Qwen3Model, optim: Any = None, step: int | None = None) -> dict:
    import torch.distributed.checkpoint as dcp

    root = Path(root)
    step = latest_iteration(root) if step is None else step
    assert step is not None, f"no checkpoint under {root}"
    d = _iter_dir(root, step)
    state: dict[str, Any] = {f"model.{k}": torch.empty_like(v, device="cpu") for k, v in mcore_state_dict(model).items()}
    if optim is not None:
        for k, v in optim.state_dict().items():
            if isinstance(v, torch.Tensor):
                state[f"optimizer.{k}"] = torch.empty_like(v, device="cpu")
    dcp.load(state, checkpoint_id=str(d))
    load_mcore_state_dict(model, {k[len("model."):]: v for k, v in state.items() if k.startswith("model.")})
    common = torch.load(d / "common.pt", weights_only=False)
    if optim is not None:
        osd = {k[len("optimizer."):]: v for k, v in state.items() if k.startswith("optimizer.")}
        osd["step"] = common.get("optimizer_step", 0)
        if "master_shard" in osd:
            osd["exp_avg"], osd["exp_avg_sq"] = osd["exp_avg"], osd["exp_avg_sq"]
        optim.load_state_dict(osd)
    return common
