"""Reshard plans for trainer -> rollout weight sync.

Reference counterpart: Megatron-Bridge ``export_hf_weights`` (all-gathers TP/EP shards
into full HF tensors) feeding ``get_named_tensor_buckets`` and the engine's
``load_weights`` (``axrl/utils/megatron/sglang_weight_updater.py:167-271``,
``axrl/utils/megatron/weight_update.py:76-100``).  Instead of gathering full tensors,
the plan maps every 128x128 tile of every *destination* shard to the one *source*
shard that holds it, so each trainer rank pushes exactly the tiles it owns.

Layout model: every fused parameter of the model is a vertical stack of logical
sub-tensors (e.g. ``qkv_proj`` = [q; k; v], ``gate_up_proj`` = [gate; up]); each
sub-tensor is split along dim 0 (column-parallel), dim 1 (row-parallel) or not at
all (replicated).  A rank's local parameter is the stack of its slices.  Flat
buffers hold all local parameters back to back (bf16 for sources; bf16 or e4m3 +
fp32 block scales for destinations).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from axrl_b200.models.qwen3 import Qwen3Config

TILE = 128


@dataclass(frozen=True)
class Sub:
    rows: int
    cols: int
    split: int  # 0 = rows (column-parallel), 1 = cols (row-parallel), -1 = replicated


@dataclass(frozen=True)
class ParamSpec:
    name: str
    subs: tuple[Sub, ...]

    def local_shape(self, tp: int) -> tuple[int, int]:
        rows = sum(s.rows // tp if s.split == 0 else s.rows for s in self.subs)
        cols = {s.cols // tp if s.split == 1 else s.cols for s in self.subs}
        assert len(cols) == 1
        return rows, cols.pop()


def qwen3_param_specs(cfg: Qwen3Config) -> list[ParamSpec]:
    """Fused parameter layout of :class:`Qwen3Model` (dense layers) in module order."""
    H, D = cfg.hidden_size, cfg.head_dim
    nq, nkv, F, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size
    specs = [ParamSpec("embed_tokens", (Sub(V, H, 0),))]
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        specs.append(ParamSpec(p + "input_layernorm.weight", (Sub(1, H, -1),)))
        if cfg.layer_is_linear(i):  # Gated DeltaNet mixer: split by heads over TP, like Megatron
            kd, vd = cfg.linear_num_key_heads * cfg.linear_key_head_dim, cfg.linear_num_value_heads * cfg.linear_value_head_dim
            nv, K = cfg.linear_num_value_heads, cfg.linear_conv_kernel_dim
            a = p + "self_attn."
            specs += [ParamSpec(a + "in_proj_qkv", (Sub(kd, H, 0), Sub(kd, H, 0), Sub(vd, H, 0))), ParamSpec(a + "in_proj_z", (Sub(vd, H, 0),)),
                      ParamSpec(a + "in_proj_b", (Sub(nv, H, 0),)), ParamSpec(a + "in_proj_a", (Sub(nv, H, 0),)),
                      ParamSpec(a + "conv_weight", (Sub(kd, K, 0), Sub(kd, K, 0), Sub(vd, K, 0))), ParamSpec(a + "dt_bias", (Sub(1, nv, 1),)),
                      ParamSpec(a + "A_log", (Sub(1, nv, 1),)), ParamSpec(a + "norm_weight", (Sub(1, cfg.linear_value_head_dim, -1),)),
                      ParamSpec(a + "out_proj", (Sub(H, vd, 1),))]
        else:
            specs += [
                ParamSpec(p + "self_attn.qkv_proj", (Sub(nq * D, H, 0), Sub(nkv * D, H, 0), Sub(nkv * D, H, 0))),
                ParamSpec(p + "self_attn.o_proj", (Sub(H, nq * D, 1),)),
                ParamSpec(p + "self_attn.q_norm", (Sub(1, D, -1),)),
                ParamSpec(p + "self_attn.k_norm", (Sub(1, D, -1),)),
            ]
            if cfg.attn_output_gate:
                specs.append(ParamSpec(p + "self_attn.attn_gate", (Sub(nq * D, H, 0),)))
        specs += [
            ParamSpec(p + "post_attention_layernorm.weight", (Sub(1, H, -1),)),
            ParamSpec(p + "mlp.gate_up_proj", (Sub(F, H, 0), Sub(F, H, 0))),
            ParamSpec(p + "mlp.down_proj", (Sub(H, F, 1),)),
        ]
    specs.append(ParamSpec("norm.weight", (Sub(1, H, -1),)))
    if not cfg.tie_word_embeddings:
        specs.append(ParamSpec("lm_head", (Sub(V, H, 0),)))
    return specs


def _align(n: int, a: int) -> int:
    return -(-n // a) * a


@dataclass
class Layout:
    """Byte offsets of each parameter inside one rank's flat buffer."""

    offsets: dict[str, int]  # element offset (source bf16) or byte offset (fp8 destination)
    scale_offsets: dict[str, int]  # byte offset of the fp32 scale grid (fp8 destination)
    shapes: dict[str, tuple[int, int]]
    nbytes: int


def build_layout(specs: list[ParamSpec], tp: int, fp8: bool, base: int = 0) -> Layout:
    """Offsets of each parameter in a flat buffer starting at byte ``base`` (256-byte aligned)."""
    assert base % 256 == 0
    offs, soffs, shapes = {}, {}, {}
    pos = base
    for s in specs:
        r, c = s.local_shape(tp)
        shapes[s.name] = (r, c)
        if not (fp8 and quantizable(s, r, c)):
            offs[s.name] = pos // 2  # bf16 element offset
            pos += _align(r * c * 2, 256)
        else:
            offs[s.name] = pos  # e4m3 byte offset, then the fp32 block-scale grid
            pos += _align(r * c, 256)
            soffs[s.name] = pos
            pos += _align(-(-r // TILE) * -(-c // TILE) * 4, 256)
    return Layout(offs, soffs, shapes, pos)


def quantizable(spec: ParamSpec, rows: int, cols: int) -> bool:
    """Block-fp8 only for TP-split matrices whose local shape is a whole number of 128x128 blocks
    (norms and other replicated vectors stay bf16) among the weights the rollout engine runs as fp8
    GEMMs (the fused attention / MLP projections)."""
    fp8_gemm = spec.name.endswith(("qkv_proj", "o_proj", "gate_up_proj", "down_proj", "lm_head", "embed_tokens"))
    return fp8_gemm and all(s.split != -1 for s in spec.subs) and rows % TILE == 0 and cols % TILE == 0


def _slices(sub: Sub, tp: int) -> list[tuple[int, int, int, int]]:
    """Per rank: (row0, row1, col0, col1) of the sub-tensor in full coordinates."""
    out = []
    for r in range(tp):
        if sub.split == 0:
            n = sub.rows // tp
            out.append((r * n, (r + 1) * n, 0, sub.cols))
        elif sub.split == 1:
            n = sub.cols // tp
            out.append((0, sub.rows, r * n, (r + 1) * n))
        else:
            out.append((0, sub.rows, 0, sub.cols))
    return out


def build_tiles(specs: list[ParamSpec], src_tp: int, dst_tp: int, src_layout: Layout, dst_layout: Layout, src_rank: int,
                dst_ranks: list[int], fp8: bool) -> np.ndarray:
    """Tiles that ``src_rank`` (TP rank of the trainer) must push to each destination TP rank.

    ``dst_ranks[j]`` is the global rank of destination TP rank j.  Returns int64 (n, 10):
    (src_off, src_ld, dst_rank, dst_off, dst_ld, rows, cols, scale_off, scale_ld, scale_idx).
    For replicated tensors only source TP rank 0 pushes.
    """
    out = []
    for ps in specs:
        sr, sc = src_layout.shapes[ps.name]
        dr, dc = dst_layout.shapes[ps.name]
        q8 = fp8 and quantizable(ps, dr, dc)
        src_row_base = 0
        dst_row_base = [0] * dst_tp
        for sub in ps.subs:
            ssl = _slices(sub, src_tp)[src_rank]
            for j in range(dst_tp):
                dsl = _slices(sub, dst_tp)[j]
                if sub.split == -1 and src_rank != 0:
                    continue
                r0, r1 = max(ssl[0], dsl[0]), min(ssl[1], dsl[1])
                c0, c1 = max(ssl[2], dsl[2]), min(ssl[3], dsl[3])
                if r0 >= r1 or c0 >= c1:
                    continue
                # local coordinates
                srow = src_row_base + r0 - ssl[0]
                scol = c0 - ssl[2]
                drow = dst_row_base[j] + r0 - dsl[0]
                dcol = c0 - dsl[2]
                for tr in range(0, r1 - r0, TILE):
                    for tc in range(0, c1 - c0, TILE):
                        rows = min(TILE, r1 - r0 - tr)
                        cols = min(TILE, c1 - c0 - tc)
                        so = src_layout.offsets[ps.name] + (srow + tr) * sc + scol + tc
                        if q8:
                            gr, gc = drow + tr, dcol + tc
                            assert gr % TILE == 0 and gc % TILE == 0, "fp8 tiles must align with 128x128 blocks"
                            do = dst_layout.offsets[ps.name] + gr * dc + gc
                            sidx = (gr // TILE) * (dc // TILE) + gc // TILE
                            out.append((so, sc, dst_ranks[j], do, dc, rows, cols, dst_layout.scale_offsets[ps.name], dc // TILE, sidx))
                        else:
                            do = dst_layout.offsets[ps.name] + (drow + tr) * dc + dcol + tc
                            out.append((so, sc, dst_ranks[j], do, dc, rows, cols, -1, 0, 0))
            # advance the stacked row bases
            src_row_base += (sub.rows // src_tp) if sub.split == 0 else sub.rows
            for j in range(dst_tp):
                dst_row_base[j] += (sub.rows // dst_tp) if sub.split == 0 else sub.rows
    return np.asarray(out, dtype=np.int64).reshape(-1, 10)


def split_modes(tiles: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(bf16-copy tiles, fp8-quantise tiles)."""
    q = tiles[:, 7] >= 0
    return tiles[~q], tiles[q]


def emulate_push(tiles: np.ndarray, src: np.ndarray, dst_bufs: dict[int, np.ndarray], fp8: bool) -> None:
    """Host reference of the push kernel (oracle for tests).  dst_bufs[rank] is a uint8/bf16 view."""
    import torch

    for t in tiles:
        so, sld, dr, do, dld, rows, cols, soff, sldd, sidx = (int(x) for x in t)
        block = np.stack([src[so + r * sld: so + r * sld + cols] for r in range(rows)])
        buf = dst_bufs[dr]
        if soff < 0:
            view = buf.view(np.uint16)
            for r in range(rows):
                view[do + r * dld: do + r * dld + cols] = block[r].view(np.uint16)
        else:
            f = torch.from_numpy(block.view(np.uint16).astype(np.int32) << 16).view(torch.float32)
            amax = max(float(f.abs().max()), 1e-12)
            q = (f * (448.0 / amax)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            for r in range(rows):
                buf[do + r * dld: do + r * dld + cols] = q[r]
            buf[soff + 4 * sidx: soff + 4 * sidx + 4] = np.frombuffer(np.float32(amax / 448.0).tobytes(), dtype=np.uint8)
