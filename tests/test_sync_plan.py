"""Weight-sync reshard plans on the host: every destination TP shard is exactly covered, bf16 tiles
reproduce the shard bit-exactly, and block-fp8 tiles dequantise within e4m3 error (kernel oracle)."""

import numpy as np
import pytest
import torch

from axrl_b200.models.qwen3 import Qwen3Config
from axrl_b200.sync.plan import _slices, build_layout, build_tiles, emulate_push, qwen3_param_specs


@pytest.mark.parametrize("src_tp,dst_tp", [(4, 2), (2, 4), (1, 2), (2, 1)])
@pytest.mark.parametrize("fp8", [False, True])
def test_reshard_plan(src_tp, dst_tp, fp8):
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=1, num_attention_heads=8,
                      num_key_value_heads=4, head_dim=128)
    specs = qwen3_param_specs(cfg)
    rng = np.random.default_rng(0)
    full = {s.name: [rng.standard_normal((sub.rows, sub.cols)).astype(np.float32) for sub in s.subs] for s in specs}

    def local(s, tp, r):
        return np.concatenate([blk[a:b, c:d] for sub, blk in zip(s.subs, full[s.name]) for a, b, c, d in [_slices(sub, tp)[r]]], 0)

    sl = build_layout(specs, src_tp, False)
    base = -(-sl.nbytes // 4096) * 4096
    dl = build_layout(specs, dst_tp, fp8, base=base)
    dst_ranks = list(range(100, 100 + dst_tp))
    bufs = {r: np.zeros(dl.nbytes, np.uint8) for r in dst_ranks}
    for r in range(src_tp):
        src = np.zeros(sl.nbytes // 2, np.uint16)
        for s in specs:
            a = torch.from_numpy(local(s, src_tp, r)).bfloat16().view(torch.int16).numpy().view(np.uint16).reshape(-1)
            src[sl.offsets[s.name]: sl.offsets[s.name] + a.size] = a
        emulate_push(build_tiles(specs, src_tp, dst_tp, sl, dl, r, dst_ranks, fp8), src, bufs, fp8)
    for j, rk in enumerate(dst_ranks):
        for s in specs:
            rr, cc = dl.shapes[s.name]
            exp = torch.from_numpy(local(s, dst_tp, j)).bfloat16().float()
            if s.name in dl.scale_offsets:
                q = torch.from_numpy(bufs[rk][dl.offsets[s.name]: dl.offsets[s.name] + rr * cc].copy()).view(torch.float8_e4m3fn).float().view(rr, cc)
                nb = (rr // 128) * (cc // 128)
                sc = torch.from_numpy(bufs[rk][dl.scale_offsets[s.name]: dl.scale_offsets[s.name] + 4 * nb].copy()).view(torch.float32)
                deq = q * sc.view(rr // 128, cc // 128).repeat_interleave(128, 0).repeat_interleave(128, 1)
                assert ((deq - exp).abs().max() / exp.abs().max()).item() < 0.07, s.name
            else:
                u = bufs[rk].view(np.uint16)[dl.offsets[s.name]: dl.offsets[s.name] + rr * cc].astype(np.int32) << 16
                assert torch.equal(torch.from_numpy(u).view(torch.float32).view(rr, cc), exp), s.name


@pytest.mark.parametrize("tp", [2, 4])
def test_specs_match_trainer_shards(tp):
    """The plan's per-rank layout of every parameter (Gated DeltaNet and gated attention included) is
    the trainer's own TP shard of it."""
    from axrl_b200.models.qwen3 import Qwen3Model
    from axrl_b200.parallel.tensor_parallel import shard_param

    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=4, head_dim=16, layer_types=["linear_attention", "full_attention"],
                      linear_num_key_heads=4, linear_num_value_heads=8, linear_key_head_dim=8, linear_value_head_dim=8,
                      attn_output_gate=True)
    m = Qwen3Model(cfg)
    m.init_weights(2)
    params = dict(m.named_parameters())
    specs = qwen3_param_specs(cfg)
    assert {s.name for s in specs} == set(params)
    for s in specs:
        full = params[s.name].detach()
        full2 = full.reshape(1, -1) if full.dim() == 1 else full
        blocks, r0 = [], 0
        for sub in s.subs:
            blocks.append(full2[r0:r0 + sub.rows])
            r0 += sub.rows
        for r in range(tp):
            want = torch.cat([blk[a:b, c:d] for sub, blk in zip(s.subs, blocks) for a, b, c, d in [_slices(sub, tp)[r]]], 0)
            got = shard_param(s.name, full, r, tp, cfg)
            torch.testing.assert_close(got.reshape(want.shape), want, msg=s.name)
