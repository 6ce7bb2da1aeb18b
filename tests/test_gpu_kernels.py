"""sm_100a kernels vs plain PyTorch fp32 references of the same ops (small shapes)."""

import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ext():
    from axrl_b200.ops import _ext

    return _ext.ext()


def close(a, b, atol, rtol=0.0, msg=""):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    lim = atol + rtol * b.abs().max().item()
    assert err <= lim, f"{msg} max err {err:.3e} > {lim:.3e}"


def test_extension_loaded_from_tree():
    from axrl_b200.ops import _ext

    m = _ext.ext()
    assert m.__file__.startswith(_ext._PKG_DIR)


@pytest.mark.parametrize("T,H", [(7, 256), (300, 4096), (64, 2048)])
def test_rmsnorm(T, H):
    from axrl_b200.ops.core import rms_norm

    x = torch.randn(T, H, device=DEV).bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16().requires_grad_(True)
    y = rms_norm(x, w, 1e-6)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    close(y, yr, 2e-2, msg="rms fwd")
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    close(x.grad, xr.grad, 3e-2, 1e-2, msg="rms dx")
    close(w.grad, wr.grad, 0.0, 2e-2, msg="rms dw")


@pytest.mark.parametrize("nq,nkv", [(4, 4), (32, 8)])
def test_qknorm_rope(nq, nkv):
    from axrl_b200.ops.core import _qk_norm_rope_ref, qk_norm_rope, rope_inv_freq

    T, D = 50, 128
    qkv = torch.randn(T, (nq + 2 * nkv) * D, device=DEV).bfloat16().requires_grad_(True)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16().requires_grad_(True)
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16().requires_grad_(True)
    pos = torch.randint(0, 30000, (T,), device=DEV, dtype=torch.int32)
    inv = rope_inv_freq(D, 1e6, DEV)
    q, k, v = qk_norm_rope(qkv, qw, kw, pos, inv, nq, nkv)
    refs = [t.detach().float().requires_grad_(True) for t in (qkv, qw, kw)]
    qr, kr, vr = _qk_norm_rope_ref(refs[0], refs[1], refs[2], pos, inv, nq, nkv, 1e-6)
    close(q, qr, 3e-2, msg="q")
    close(k, kr, 3e-2, msg="k")
    close(v, vr, 0.0, msg="v")
    gq, gk, gv = torch.randn_like(qr), torch.randn_like(kr), torch.randn_like(vr)
    torch.autograd.backward([q, k, v], [gq.bfloat16(), gk.bfloat16(), gv.bfloat16()])
    torch.autograd.backward([qr, kr, vr], [gq, gk, gv])
    close(qkv.grad, refs[0].grad, 5e-2, 1e-2, msg="dqkv")
    close(qw.grad, refs[1].grad, 0.0, 3e-2, msg="dqw")
    close(kw.grad, refs[2].grad, 0.0, 3e-2, msg="dkw")


def test_swiglu():
    from axrl_b200.ops.core import swiglu

    gu = torch.randn(33, 2 * 768, device=DEV).bfloat16().requires_grad_(True)
    y = swiglu(gu)
    r = gu.detach().float().requires_grad_(True)
    g, u = r.chunk(2, -1)
    yr = torch.nn.functional.silu(g) * u
    close(y, yr, 2e-2, 1e-2)
    d = torch.randn_like(yr)
    y.backward(d.bfloat16())
    yr.backward(d)
    close(gu.grad, r.grad, 3e-2, 1e-2)


@pytest.mark.parametrize("M,N,K", [(1, 512, 256), (37, 768, 1024), (200, 1024, 512), (1024, 2048, 4096), (4096, 6144, 4096)])
def test_gemm_family(M, N, K):
    e = _ext()
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    y = e.linear_fwd(x, w)
    close(y, x.float() @ w.float().T, 2e-2, 1e-2, msg="fwd")
    dy = torch.randn(M, N, device=DEV).bfloat16()
    close(e.linear_dgrad(dy, w), dy.float() @ w.float(), 3e-2, 1e-2, msg="dgrad")
    ref = dy.float().T @ x.float()
    close(e.linear_wgrad(dy, x), ref, 0.0, 1.5e-2, msg="wgrad")
    acc = torch.ones(N, K, device=DEV)
    e.linear_wgrad_acc(dy, x, acc)
    close(acc, ref + 1, 1e-3, 1e-3, msg="wgrad acc")


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100])
@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 12288), (24576, 4096), (1024, 256), (65600, 128)])
def test_linear_residual_and_skinny(M, N, K):
    """Decode-shaped GEMMs: skinny weight-streaming kernel (M <= 64, split-K with self-cleaning
    workspace, no split when M x N exceeds it) and the residual-fused epilogue; called twice to
    check the workspace is left clean."""
    e = _ext()
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    ref = x.float() @ w.float().T
    for _ in range(2):
        close(e.linear_fwd(x, w), ref, 2e-2, 1e-2, msg="fwd")
        close(e.linear_residual(x, w, r), ref + r.float(), 3e-2, 1e-2, msg="fwd+residual")
        if M <= 64:
            for v in ("skinny", "swapab"):
                close(e.linear_variant(x, w, v), ref, 2e-2, 1e-2, msg=v)


def _spec_cases():
    from axrl_b200.data import prefix_tree as pt
    from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens, tree_spec

    cases = [causal_spec_from_cu_seqlens([0, 5, 130, 131, 400]), causal_spec_from_cu_seqlens([0, 1000])]
    paths = [[1] * 150 + [2] * 70, [1] * 150 + [3] * 33, [1] * 90]
    packed, nodes, _ = pt.build_tree_packed_sequence(paths)
    q, k, t = pt.build_prefix_tree_ranges_as_lists(nodes)
    cases.append(tree_spec(q, k, t, len(packed)))
    return cases


@pytest.mark.parametrize("case", [0, 1, 2])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2)])
def test_attention(case, hq, hkv):
    from axrl_b200.ops.core import _attn_ref, attention

    spec = _spec_cases()[case]
    T, D = spec.total_q, 128
    torch.manual_seed(case)
    q = torch.randn(T, hq, D, device=DEV).bfloat16().requires_grad_(True)
    k = torch.randn(T, hkv, D, device=DEV).bfloat16().requires_grad_(True)
    v = torch.randn(T, hkv, D, device=DEV).bfloat16().requires_grad_(True)
    o = attention(q, k, v, spec)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    orf = _attn_ref(qr, kr, vr, spec, 1 / math.sqrt(D))
    close(o, orf, 2e-2, msg="attn fwd")
    g = torch.randn_like(orf)
    o.backward(g.bfloat16())
    orf.backward(g)
    close(q.grad, qr.grad, 5e-2, 2e-2, msg="dq")
    close(k.grad, kr.grad, 5e-2, 2e-2, msg="dk")
    close(v.grad, vr.grad, 5e-2, 2e-2, msg="dv")


@pytest.mark.parametrize("ent", [False, True])
def test_fused_logprob(ent):
    from axrl_b200.ops.logprob import fused_logprob, logprob_ref

    T, H, V = 300, 256, 5000
    h = torch.randn(T, H, device=DEV).bfloat16().requires_grad_(True)
    w = (torch.randn(V, H, device=DEV) / 16).bfloat16().requires_grad_(True)
    lab = torch.randint(0, V, (T,), device=DEV)
    lab[::7] = -100
    lp, e = fused_logprob(h, w, lab, temperature=0.7, compute_entropy=ent, chunk=128)
    hr, wr = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lpr, er = logprob_ref(hr, wr, lab, 0.7, ent)
    lpr = torch.where(lab >= 0, lpr, torch.zeros_like(lpr))
    close(lp, lpr, 5e-2, msg="lp")
    gl = torch.randn(T, device=DEV)
    loss = (lp * gl).sum()
    loss_r = (lpr * gl).sum()
    if ent:
        close(e, er, 5e-2, msg="entropy")
        ge = torch.randn(T, device=DEV)
        loss = loss + (e * ge).sum()
        loss_r = loss_r + (er * ge).sum()
    loss.backward()
    loss_r.backward()
    close(h.grad, hr.grad, 0.0, 5e-2, msg="dh")
    close(w.grad, wr.grad, 0.0, 5e-2, msg="dw")


def test_sampler():
    from axrl_b200.ops.paged import sample

    B, V = 64, 1000
    logits = torch.randn(B, V, device=DEV) * 3
    temp = torch.ones(B, device=DEV)
    temp[:8] = 0.0  # greedy rows
    seed = torch.tensor([123], device=DEV)
    forced = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    forced[10] = 5
    tok, lp = sample(logits.bfloat16(), temp, seed, forced=forced, row_ids=torch.arange(B, device=DEV, dtype=torch.int32))
    lb = logits.bfloat16().float()
    assert torch.equal(tok[:8], lb[:8].argmax(-1))
    assert tok[10].item() == 5
    ref_lp = torch.log_softmax(lb, -1).gather(1, tok[:, None]).squeeze(1)
    close(lp[8:], ref_lp[8:], 1e-3)
    # distribution check on one row with a small vocabulary
    small = torch.tensor([[0.0, 1.0, 2.0, -1.0]], device=DEV).repeat(20000, 1)
    t2, _ = sample(small, torch.ones(20000, device=DEV), seed, row_ids=torch.arange(20000, device=DEV, dtype=torch.int32))
    freq = torch.bincount(t2, minlength=4).float() / 20000
    close(freq, torch.softmax(small[0], -1), 0.02, msg="sampling frequencies")


@pytest.mark.parametrize("planned_kernel", ["tma", "persist"])
def test_paged_decode_attention(planned_kernel):
    """Fixed-grid split-KV kernel, then the planned work-list kernels (the TMA page pipeline, the
    default, and the cp.async persistent kernel) after in-place length changes."""
    from axrl_b200.ops.paged import DecodeWorkspace, decode_attention_ref, paged_decode_attention

    _ext().set_decode_attn_tma(planned_kernel == "tma")

    B, Hq, Hkv, D, P, pages = 5, 32, 8, 128, 64, 64
    kc = torch.randn(pages, Hkv, P, D, device=DEV).bfloat16()
    vc = torch.randn(pages, Hkv, P, D, device=DEV).bfloat16()
    lens = torch.tensor([1, 63, 64, 700, 1500], dtype=torch.int32, device=DEV)
    bt = torch.zeros(B, 40, dtype=torch.int32, device=DEV)
    perm = torch.randperm(pages, device=DEV)
    off = 0
    for b in range(B):
        n = (int(lens[b]) + P - 1) // P
        bt[b, :n] = perm[off:off + n] % pages
        off = (off + n) % 40
    q = torch.randn(B, Hq, D, device=DEV).bfloat16()
    ws = DecodeWorkspace(B, Hq, 40 * P, DEV)
    o = paged_decode_attention(q, kc, vc, bt, lens, ws)
    r = decode_attention_ref(q, kc, vc, bt, lens, 1 / math.sqrt(D))
    close(o, r, 2e-2)
    # persistent work-list kernel after an in-place length change (plan once, reuse per layer)
    lens.copy_(torch.tensor([129, 2, 2500, 0 + 1, 640], dtype=torch.int32, device=DEV))
    for b in range(B):
        n = (int(lens[b]) + P - 1) // P
        bt[b, :n] = torch.randint(0, pages, (n,), device=DEV, dtype=torch.int32)
    ws.plan(lens)
    for _ in range(2):
        o = paged_decode_attention(q, kc, vc, bt, lens, ws, planned=True)
        close(o, decode_attention_ref(q, kc, vc, bt, lens, 1 / math.sqrt(D)), 2e-2)
    assert ws.prefix[:B + 1].tolist() == [0, 2, 3, 23, 24, 29]
    _ext().set_decode_attn_tma(True)


def test_adamw_and_sqnorm():
    e = _ext()
    n = 10_003
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    pb = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    sq = torch.zeros(1, device=DEV)
    e.sqnorm_accumulate(g, sq)
    close(sq, g.pow(2).sum()[None], 0.0, 1e-4)
    p0 = p.clone()
    e.adamw_step(p, g, m, v, pb, 5000, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1, sq, 1.0, 0.5)
    gn = (sq.sqrt() * 0.5).item()
    gs = 0.5 * min(1.0, 1.0 / (gn + 1e-6))
    gg = g * gs
    mr = 0.1 * gg
    vr = 0.001 * gg * gg
    upd = (mr / 0.1) / ((vr / 0.001).sqrt() + 1e-8)
    upd[:5000] += 0.01 * p0[:5000]
    close(p, p0 - 1e-3 * upd, 1e-6, 1e-5)
    # the bf16 copy is the fp32 master rounded to bf16 (within one bf16 ulp, 2^-7 relative)
    torch.testing.assert_close(pb.float(), p.bfloat16().float(), atol=0.0, rtol=8e-3)


def test_embedding():
    from axrl_b200.ops.core import embedding

    table = torch.randn(100, 256, device=DEV).bfloat16().requires_grad_(True)
    ids = torch.randint(0, 100, (77,), device=DEV)
    out = embedding(ids, table)
    assert torch.equal(out, table.detach()[ids])
    g = torch.randn_like(out, dtype=torch.float32)
    out.backward(g.bfloat16())
    ref = torch.zeros(100, 256, device=DEV).index_add_(0, ids, g.bfloat16().float())
    close(table.grad, ref, 2e-2)


def test_grouped_linear_fwd_bwd_matches_per_expert_fp32():
    """One grouped tcgen05 GEMM over all experts (device offsets, some experts empty) against
    per-expert fp32 matmuls; dgrad and the fp32 wgrad accumulation into main_grad."""
    from axrl_b200.ops.grouped import expert_offsets, grouped_linear

    torch.manual_seed(0)
    E, N, K = 6, 384, 256
    ids = torch.tensor([0] * 70 + [2] * 1 + [3] * 200 + [5] * 33, device="cuda")
    off = expert_offsets(ids, E)
    M = ids.numel()
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(E, N, K, device="cuda") * 0.05).bfloat16().requires_grad_(True)
    w.main_grad = torch.ones(E, N, K, device="cuda")  # accumulates on top
    y = grouped_linear(x, w, off)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    y.backward(dy)
    o = off.tolist()
    xf, wf, dyf = x.detach().float(), w.detach().float(), dy.float()
    for e in range(E):
        r0, r1 = o[e], o[e + 1]
        if r1 > r0:
            torch.testing.assert_close(y[r0:r1].float(), xf[r0:r1] @ wf[e].t(), atol=3e-2, rtol=2e-2)
            torch.testing.assert_close(x.grad[r0:r1].float(), dyf[r0:r1] @ wf[e], atol=3e-2, rtol=2e-2)
        exp = 1.0 + dyf[r0:r1].t() @ xf[r0:r1]
        torch.testing.assert_close(w.main_grad[e], exp, atol=5e-2, rtol=2e-2)
    assert w.grad is None


@pytest.mark.parametrize("dual", [None, 3.0])
def test_fused_grpo_policy_loss_matches_torch(dual):
    """Fused per-token GRPO/PPO objective (ratio, clip, dual clip, IS weight, gradient) against the
    PyTorch oracle of GrpoTrainer.grpo_loss, values and d loss / d logprobs."""
    from axrl_b200.configs import GrpoTrainerConfig
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer

    torch.manual_seed(1)
    B, S = 6, 300
    lp = (-torch.rand(B, S) * 3).double()
    base = lp + torch.randn(B, S) * 0.3
    base[0, :5] = lp[0, :5] + 30  # log-ratio clamp region
    adv = torch.randn(B, S)
    adv[1] = 0.0
    w = torch.rand(B, S) * 2
    mask = torch.rand(B, S) > 0.2
    t = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo", clip_ratio_low=0.2, clip_ratio_high=0.28, dual_clip_neg_adv_factor=dual,
                                      loss_agg_type="token-mean"))
    outs = {}
    for dev in ("cpu", "cuda"):
        x = lp.float().to(dev).requires_grad_(True)
        loss, ratio, eff = t.grpo_loss(loss_mask=mask.to(dev), advantages=adv.to(dev), logprobs=x, base_logprobs=base.float().to(dev),
                                       token_mismatch_tir=w.to(dev))
        loss.backward()
        outs[dev] = (loss.detach().cpu(), x.grad.cpu(), ratio.detach().cpu(), eff.detach().cpu())
    for a, b in zip(outs["cpu"], outs["cuda"]):
        torch.testing.assert_close(b, a, atol=1e-5, rtol=1e-4)


def test_fp8_block_linear_matches_dequantized_fp32():
    """Block-scaled e4m3 GEMM (1x128 activation scales, 128x128 weight scales) against the fp32
    product of the dequantised operands, and the activation quantiser against its torch oracle."""
    from axrl_b200.ops import _ext
    from axrl_b200.ops.fp8 import Fp8Weight, dequantize_weight_blocks, fp8_linear, quantize_rows_ref

    torch.manual_seed(0)
    for M, N, K in [(8, 256, 512), (200, 384, 1024), (1000, 1024, 256)]:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
        fw = Fp8Weight.from_dense(w)
        xq, xs = _ext.ext().quant_fp8_rows(x)
        rq, rs = quantize_rows_ref(x)
        torch.testing.assert_close(xs, rs, atol=0, rtol=1e-6)
        # the kernel multiplies by 1/scale, the oracle divides: rare one-step rounding differences
        assert (xq.float() != rq.float()).float().mean().item() < 0.01
        y = fp8_linear(x, fw).float()
        ref = (xq.float() * xs.repeat_interleave(128, 1)) @ dequantize_weight_blocks(fw.q, fw.s).t()
        torch.testing.assert_close(y, ref, atol=2e-2, rtol=2e-2)
        dense = x.float() @ w.float().t()  # quantisation error stays small
        assert ((y - dense).norm() / dense.norm()).item() < 0.08


def test_rollout_engine_fp8_weights_run():
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine

    cfg = Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128)
    m = Qwen3Model(cfg)
    m.init_weights(0)
    m = m.to("cuda", torch.bfloat16)
    m.inv_freq = m.inv_freq.float()
    eng = RolloutEngine(m, max_batch=4, kv_tokens=2048, max_context=256, seed=0, weight_format="fp8_block")
    assert len(eng.fp8) == 4 * cfg.num_hidden_layers // 2 * 2
    res = eng.generate([GenRequest(rid=f"r{i}", prompt=list(range(5, 40)), max_new_tokens=20, seed_stream=i) for i in range(3)])
    assert all(len(r.output_ids) == 20 and all(lp <= 0 for lp in r.output_logprobs) for r in res)
    eng.release_graphs()


def test_bounded_flag_wait_times_out_and_context_stays_usable():
    """A device-side wait on a flag that nothing sets gives up after its limit, reports status 1,
    and the CUDA context keeps working (no trap, no hang)."""
    import time

    from axrl_b200.ops import _ext

    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    _ext.ext().flag_wait_bounded(flags, 3, 7, 50_000_000, status)  # 50 ms limit
    torch.cuda.synchronize()
    assert status.item() == 1 and time.time() - t0 < 5
    flags[3] = 7
    _ext.ext().flag_wait_bounded(flags, 3, 7, 50_000_000, status)
    torch.cuda.synchronize()
    assert status.item() == 0 and flags[3].item() == 0  # consumed
    assert (torch.ones(4, device="cuda") * 2).sum().item() == 8


def test_fused_logprob_topk_entropy_and_argmax():
    """Top-k masked entropy (values and gradients w.r.t. hidden and weight) against the fp32 oracle."""
    from axrl_b200.ops.logprob import argmax_tokens, fused_logprob, logprob_ref

    torch.manual_seed(3)
    T, H, V = 300, 256, 4096
    h = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(V, H, device="cuda") * 0.05).bfloat16().requires_grad_(True)
    lab = torch.randint(0, V, (T,), device="cuda")
    lp, ent = fused_logprob(h, w, lab, temperature=0.8, compute_entropy=True, entropy_top_k=20, chunk=128)
    (lp.sum() + 3.0 * ent.sum()).backward()
    hr, wr = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lpr, entr = logprob_ref(hr, wr, lab, temperature=0.8, compute_entropy=True, entropy_top_k=20)
    (lpr.sum() + 3.0 * entr.sum()).backward()
    torch.testing.assert_close(lp, lpr, atol=3e-2, rtol=0)
    torch.testing.assert_close(ent, entr, atol=3e-2, rtol=0)
    assert ((h.grad.float() - hr.grad).norm() / hr.grad.norm()).item() < 3e-2
    assert ((w.grad.float() - wr.grad).norm() / wr.grad.norm()).item() < 3e-2
    am = argmax_tokens(h.detach(), w.detach())
    ref = (h.detach().float() @ w.detach().float().t()).argmax(-1)
    assert (am == ref).float().mean().item() > 0.98


@pytest.mark.parametrize("renorm", [True, False])
def test_fused_router_matches_torch(renorm):
    """Softmax + top-k + replay + renorm kernel and its backward against the PyTorch routing."""
    from axrl_b200.models import moe

    torch.manual_seed(0)
    T, E, k = 500, 128, 8
    x = torch.randn(T, E, device="cuda")
    replay = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)])
    mask = torch.rand(T, device="cuda") < 0.5
    for rp, rm in ((None, None), (replay, mask)):
        a = x.clone().requires_grad_(True)
        b = x.clone().requires_grad_(True)
        w1, i1 = moe.route(a, k, renorm, rp, rm)
        w2, i2 = moe.route(b.cpu(), k, renorm, None if rp is None else rp.cpu(), None if rm is None else rm.cpu())
        assert torch.equal(i1.cpu(), i2)
        torch.testing.assert_close(w1.cpu(), w2, atol=1e-6, rtol=1e-5)
        gw = torch.randn(T, k)
        w1.backward(gw.cuda())
        w2.backward(gw)
        torch.testing.assert_close(a.grad.cpu(), b.grad.cpu(), atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("M", [1, 5, 16, 23, 32])
def test_skinny_tma_gemm_matches_fp32(M):
    """TMA-fed weight-streaming GEMM (persistent CTAs, mbarrier ring, split tiles with a
    self-cleaning workspace) against fp32, including N not a multiple of the 128-row tile."""
    from axrl_b200.ops import _ext

    torch.manual_seed(M)
    e = _ext.ext()
    for N, K in [(4096, 4096), (6144, 4096), (200, 512), (1032, 12288)]:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        ref = x.float() @ w.float().t()
        for _ in range(2):  # the workspace must be clean again after each call
            y = e.linear_variant(x, w, "tma")
            torch.testing.assert_close(y.float(), ref, atol=2e-2, rtol=2e-2)
    assert e.skinny_tma_error() == 0


@pytest.mark.parametrize("variant", ["skinny", "tma", "tccluster"])
def test_decode_gemm_chain_with_programmatic_launch(variant):
    """Decode-size GEMMs launched with programmatic dependent launch and early weight loads: each
    GEMM must read the activation its predecessor (RMSNorm) just wrote, add the residual that an
    earlier GEMM wrote, and write into caller-provided rows; checked against fp32 over a chain of
    dependent launches with changing data."""
    e = _ext()
    torch.manual_seed(3)
    H, N = 1024, 1536
    w1 = (torch.randn(N, H, device=DEV) * 0.03).bfloat16()
    w2 = (torch.randn(H, N, device=DEV) * 0.03).bfloat16()
    g = torch.ones(H, device=DEV).bfloat16()
    e.set_pdl(True)
    e.set_weights_static(True)
    if variant == "tccluster":
        e.set_decode_gemm("tccluster")
    try:
        for M in (1, 8, 13) + ((40, 64) if variant == "tccluster" else ()):
            h = torch.randn(M, H, device=DEV).bfloat16()
            for _ in range(4):
                x = e.rmsnorm_fwd(h, g, 1e-6)[0]
                y = e.linear_variant(x, w1, variant) if variant == "tma" else e.linear_fwd(x, w1)
                out = torch.empty(M, H, device=DEV, dtype=torch.bfloat16)
                e.linear_fwd_into(y, w2, out)
                h2 = e.linear_residual(y, w2, h)
                xr = h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-6)
                yr = xr.bfloat16().float() @ w1.float().t()
                close(y, yr, 3e-2, 2e-2, msg=f"first GEMM M={M}")
                o_ref = y.float() @ w2.float().t()
                close(out, o_ref, 3e-2, 2e-2, msg=f"GEMM into rows M={M}")
                close(h2, o_ref + h.float(), 3e-2, 2e-2, msg=f"residual GEMM M={M}")
                h = h2
    finally:
        e.set_weights_static(False)
        e.set_decode_gemm("")
    torch.cuda.synchronize()
    assert e.skinny_tma_error() == 0 and e.tc_stream_error() == 0


@pytest.mark.parametrize("variant", [0, 2, 3, 4,
    pytest.param(1, marks=pytest.mark.skipif(
        os.environ.get("AXRL_TEST_ATTN_TC2") != "1", reason="double-buffered-P variant: gives NaN on some inputs, under investigation"))])
@pytest.mark.parametrize("case", [0, 1, 2, 3, 4])
def test_attention_tcgen05_forward_matches_reference(case, variant):
    """tcgen05/TMEM/TMA forward (attention_tc.cu) against fp32 and the mma.sync kernel: causal
    packs with odd lengths, a prefix tree, full (non-causal) ranges, keys gathered from a longer
    buffer than the queries (context-parallel layout), and sharp scores that make the running
    maximum jump (O rescaled in TMEM)."""
    from axrl_b200.ops.attention_spec import spec_from_triples
    from axrl_b200.ops.core import _attn_ref

    e = _ext()
    D = 128
    if case < 3:
        spec = _spec_cases()[case]
        hq, hkv, sharp = 8, 2, 1.0
    elif case == 3:  # full ranges + a causal one, keys from a longer buffer
        spec = spec_from_triples([(0, 200, 0, 300, 0), (200, 457, 300, 557, 1), (457, 600, 100, 250, 0)], 600, total_k=700)
        hq, hkv, sharp = 4, 4, 1.0
    else:  # a long causal sequence with sharp scores
        from axrl_b200.ops.attention_spec import causal_spec_from_cu_seqlens

        spec = causal_spec_from_cu_seqlens([0, 77, 2100])
        hq, hkv, sharp = 8, 1, 6.0
    spec = spec.to(DEV)
    T, Tk = spec.total_q, spec.total_k
    torch.manual_seed(100 + case)
    q = (torch.randn(T, hq, D, device=DEV) * sharp).bfloat16()
    k = torch.randn(Tk, hkv, D, device=DEV).bfloat16()
    v = torch.randn(Tk, hkv, D, device=DEV).bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = e.attn_fwd_tc(q, k, v, spec.qseg, spec.kr, spec.fwd_tiles, scale, variant)
    o2, lse2 = e.attn_fwd_mma(q, k, v, spec.qseg, spec.kr, spec.fwd_tiles, scale)
    torch.cuda.synchronize()
    assert e.attn_tc_error() == 0
    if Tk == T:
        close(o, _attn_ref(q.float(), k.float(), v.float(), spec, scale), 2e-2, msg="tc vs fp32")
    close(o, o2, 4e-2, msg="tc vs mma.sync")  # each within 2e-2 of fp32 (bf16 P rounding)
    fin = torch.isfinite(lse2)
    assert torch.equal(fin, torch.isfinite(lse)), "rows without keys differ"
    close(lse[fin], lse2[fin], 1e-3, 1e-4, msg="lse")


@pytest.mark.parametrize("variant", ["tile128", "blocks64", "dbl"])
@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_attention_tcgen05_backward_matches_mma(case, variant):
    """tcgen05 backward (attention_tc_bwd.cu; 128-row q tiles, the same with Q / dO double-buffered
    and P^T in tensor memory, or 64-row blocks through a 3-stage ring with dQ^T read out by separate
    warps) against the mma.sync backward on the same inputs:
    causal packs, a prefix tree, full ranges with a longer key buffer."""
    from axrl_b200.ops.attention_spec import spec_from_triples

    e = _ext()
    D = 128
    if case < 3:
        spec, hq, hkv = _spec_cases()[case], 8, 2
    else:
        spec, hq, hkv = spec_from_triples([(0, 200, 0, 300, 0), (200, 457, 300, 557, 1)], 457, total_k=600), 4, 4
    spec = spec.to(DEV)
    T, Tk = spec.total_q, spec.total_k
    torch.manual_seed(7 + case)
    q = torch.randn(T, hq, D, device=DEV).bfloat16()
    k = torch.randn(Tk, hkv, D, device=DEV).bfloat16()
    v = torch.randn(Tk, hkv, D, device=DEV).bfloat16()
    do = torch.randn(T, hq, D, device=DEV).bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = e.attn_fwd_mma(q, k, v, spec.qseg, spec.kr, spec.fwd_tiles, scale)
    e.set_attn_bwd_tc(False)
    try:
        ref = e.attn_bwd(do, q, k, v, o, lse, spec.kseg, spec.qr, spec.bwd_tiles, scale, spec.bwd_tiles_tc)
    finally:
        e.set_attn_bwd_tc(True)
    e.set_attn_bwd_blocks64(variant == "blocks64")
    e.set_attn_bwd_dbl(variant == "dbl")
    try:
        got = e.attn_bwd(do, q, k, v, o, lse, spec.kseg, spec.qr, spec.bwd_tiles, scale, spec.bwd_tiles_tc)
        torch.cuda.synchronize()
    finally:
        e.set_attn_bwd_blocks64(False)
        e.set_attn_bwd_dbl(True)  # the default
    assert e.attn_bwd_tc_error() == 0
    for name, a, b in zip(("dq", "dk", "dv"), got, ref):
        close(a, b, 3e-2, 2e-2, msg=name)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_attention_deterministic_dq(case):
    """Deterministic mode: dQ from one CTA per q tile (no atomics) equals the atomic path and is
    bitwise reproducible."""
    e = _ext()
    D = 128
    spec = _spec_cases()[case].to(DEV)
    T = spec.total_q
    torch.manual_seed(11 + case)
    q = torch.randn(T, 8, D, device=DEV).bfloat16()
    k = torch.randn(T, 2, D, device=DEV).bfloat16()
    v = torch.randn(T, 2, D, device=DEV).bfloat16()
    do = torch.randn(T, 8, D, device=DEV).bfloat16()
    scale = 1 / math.sqrt(D)
    o, lse = e.attn_fwd_mma(q, k, v, spec.qseg, spec.kr, spec.fwd_tiles, scale)
    args = (do, q, k, v, o, lse, spec.kseg, spec.qr, spec.bwd_tiles, scale, spec.bwd_tiles_tc, spec.qseg, spec.kr, spec.fwd_tiles)
    ref = e.attn_bwd(*args)
    e.set_attn_deterministic(True)
    try:
        a, b = e.attn_bwd(*args), e.attn_bwd(*args)
    finally:
        e.set_attn_deterministic(False)
    for x, y in zip(a, b):
        assert torch.equal(x, y), "deterministic backward is not reproducible"
    for name, x, y in zip(("dq", "dk", "dv"), a, ref):
        close(x, y, 2e-2, 1e-2, msg=name)


def test_gdn_step_kernel_matches_reference():
    from axrl_b200.models.gdn import gated_delta_step

    e = _ext()
    torch.manual_seed(0)
    B, H, dk, dv, slots_n = 5, 4, 128, 128, 9
    q = torch.nn.functional.normalize(torch.randn(B, H, dk, device=DEV), dim=-1) / dk ** 0.5
    k = torch.nn.functional.normalize(torch.randn(B, H, dk, device=DEV), dim=-1)
    v, g, beta = torch.randn(B, H, dv, device=DEV), -torch.rand(B, H, device=DEV), torch.rand(B, H, device=DEV)
    pool = torch.randn(slots_n, H, dk, dv, device=DEV) * 0.1
    slots = torch.tensor([3, 0, 7, 1, 8], device=DEV)
    S = pool[slots].clone()
    o_ref, S_ref = gated_delta_step(q, k, v, g, beta, S)
    o = e.gdn_step(q, k, v, g, beta, pool, slots)
    close(o, o_ref, 1e-4, 1e-4, msg="o")
    close(pool[slots], S_ref, 1e-4, 1e-4, msg="state")


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 256), (4096, 4096, 4096), (1000, 6144, 4096), (77, 1056, 128)])
def test_tcgemm_matches_fp32(M, N, K):
    """Persistent tcgen05 GEMM (tcgemm.cu) against fp32: ragged M, N a multiple of 32 but not of
    the 256-column tile, several tiles per CTA, with and without a residual."""
    e = _ext()
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    ref = x.float() @ w.float().t()
    y = e.tc_linear(x, w)
    y2 = e.tc_linear(x, w, r)
    torch.cuda.synchronize()
    assert e.tc_linear_error() == 0
    close(y, ref, 2e-2, 1e-2, msg="tcgemm")
    close(y2, ref + r.float(), 3e-2, 1e-2, msg="tcgemm + residual")


@pytest.mark.skipif(os.environ.get("AXRL_TEST_TCGEMM") != "1", reason="tcgen05 weight-streaming GEMM: opt-in until validated on a B200")
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (17, 6144, 4096), (32, 4096, 12288), (33, 1000, 512), (64, 24576, 4096), (64, 4096, 64)])
def test_tcgemm_stream_matches_fp32(M, N, K):
    """Decode-size GEMM streaming the weights on tcgen05: split-K partials through the self-cleaning
    workspace (several calls in a row) and whole-tile direct stores, with a residual."""
    e = _ext()
    torch.manual_seed(M * 7 + N)
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    for it in range(3):
        x = torch.randn(M, K, device=DEV).bfloat16()
        r = torch.randn(M, N, device=DEV).bfloat16()
        ref = x.float() @ w.float().t()
        y = e.tc_stream_linear(x, w)
        y2 = e.tc_stream_linear(x, w, r)
        torch.cuda.synchronize()
        assert e.tc_stream_error() == 0
        close(y, ref, 2e-2, 1e-2, msg=f"tcstream call {it}")
        close(y2, ref + r.float(), 3e-2, 1e-2, msg=f"tcstream + residual call {it}")


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (8, 6144, 4096), (16, 1000, 512), (17, 6144, 4096), (32, 4096, 12288),
                                   (48, 24576, 4096), (64, 4096, 64), (64, 50000, 1024), (65, 6144, 4096), (128, 4096, 12288),
                                   (100, 1000, 512)])
def test_tcgemm_stream_cluster_matches_fp32(M, N, K):
    """Decode-size GEMM streaming the weights on tcgen05 with the split-K partials reduced inside a
    thread-block cluster: against fp32, with and without the residual, bit-identical across calls."""
    e = _ext()
    torch.manual_seed(M * 5 + N)
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    e.set_decode_gemm("tccluster")
    try:
        for it in range(2):
            x = torch.randn(M, K, device=DEV).bfloat16()
            r = torch.randn(M, N, device=DEV).bfloat16()
            ref = x.float() @ w.float().t()
            y = e.linear_fwd(x, w)
            y_again = e.linear_fwd(x, w)
            y2 = e.linear_residual(x, w, r)
            torch.cuda.synchronize()
            assert e.tc_stream_error() == 0
            close(y, ref, 2e-2, 1e-2, msg=f"tccluster call {it}")
            close(y2, ref + r.float(), 3e-2, 1e-2, msg=f"tccluster + residual call {it}")
            assert torch.equal(y, y_again), "cluster reduction must be deterministic"
    finally:
        e.set_decode_gemm("")


@pytest.mark.parametrize("M", [1, 8, 17, 40, 64, 96, 128])
def test_streaming_gemm_with_folded_rmsnorm_and_swiglu(M):
    """RMSNorm folded into the weight-streaming GEMM (per-token 1/rms applied after the cluster
    reduction) and SwiGLU folded into it (gate and up slabs combined in shared memory), against fp32
    compositions of the separate ops, with and without the residual."""
    e = _ext()
    torch.manual_seed(100 + M)
    K, N, F = 4096, 6144, 1536
    h = (torch.randn(M, K, device=DEV) * 3).bfloat16()
    g = (1 + 0.1 * torch.randn(K, device=DEV)).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.02).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    hf = h.float()
    xn = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * g.float()
    ref = xn @ w.float().t()
    y = e.linear_rms_stream(h, g, 1e-6, w)
    y2 = e.linear_rms_stream(h, g, 1e-6, w, r)
    gu = torch.randn(M, 2 * F, device=DEV).bfloat16()
    wd = (torch.randn(K, F, device=DEV) * 0.03).bfloat16()
    rd = torch.randn(M, K, device=DEV).bfloat16()
    gf, uf = gu.float()[:, :F], gu.float()[:, F:]
    ref_d = (gf * torch.sigmoid(gf) * uf) @ wd.float().t()
    yd = e.linear_swiglu_stream(gu, wd)
    yd2 = e.linear_swiglu_stream(gu, wd, rd)
    torch.cuda.synchronize()
    assert e.tc_stream_error() == 0
    close(y, ref, 3e-2, 2e-2, msg="rms-folded GEMM")
    close(y2, ref + r.float(), 4e-2, 2e-2, msg="rms-folded GEMM + residual")
    close(yd, ref_d, 3e-2, 2e-2, msg="swiglu-folded GEMM")
    close(yd2, ref_d + rd.float(), 4e-2, 2e-2, msg="swiglu-folded GEMM + residual")


@pytest.mark.parametrize("M,N,K", [(512, 256, 128), (1000, 4096, 1024), (4096, 6144, 4096), (777, 512, 96)])
def test_tcgemm_dgrad_wgrad_match_fp32(M, N, K):
    """Data gradient (W read MN-major) and fp32 weight-gradient accumulation (both operands MN-major,
    ragged token count) on the hand-written tcgen05 GEMM, against fp32."""
    e = _ext()
    torch.manual_seed(M + K)
    dy = torch.randn(M, N, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    x = torch.randn(M, K, device=DEV).bfloat16()
    dx = e.tc_linear_dgrad(dy, w)
    acc = torch.randn(N, K, device=DEV)
    acc0 = acc.clone()
    e.tc_linear_wgrad_acc(dy, x, acc, True)
    g = torch.empty(N, K, device=DEV)
    e.tc_linear_wgrad_acc(dy, x, g, False)
    torch.cuda.synchronize()
    assert e.tc_linear_error() == 0
    close(dx, dy.float() @ w.float(), 2e-2, 1e-2, msg="dgrad")
    ref = dy.float().t() @ x.float()
    close(g, ref, 1e-2, 1e-3, msg="wgrad")
    close(acc, acc0 + ref, 1e-2, 1e-3, msg="wgrad accumulate")


def test_adamw_fused_with_parameter_store_matches_unfused():
    """Partitioned AdamW fused with the bf16 parameter store (the distributed optimizer's update +
    all-gather kernel), here with this GPU's own buffer as the only destination: same masters,
    moments and bf16 parameters as the AdamW kernel with its bf16 write-back."""
    e = _ext()
    n, s0 = 40_000, 1024
    g = torch.randn(n, device=DEV)
    outs = []
    for fused in (False, True):
        torch.manual_seed(3)
        p = torch.randn(n, device=DEV)
        m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
        params = torch.zeros(s0 + n, dtype=torch.bfloat16, device=DEV)
        sq = (g.pow(2).sum() * 4.0).reshape(1)
        for step in (1, 2):
            if fused:
                ptrs = torch.tensor([params.data_ptr()], dtype=torch.int64, device=DEV)
                e.adamw_p2p_step(p, g, m, v, ptrs, s0, 30_000, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, sq, 1.0, 0.5)
            else:
                e.adamw_step(p, g, m, v, params[s0:], 30_000, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, sq, 1.0, 0.5)
        torch.cuda.synchronize()
        outs.append((p, m, v, params))
    for a, b in zip(outs[0][:3], outs[1][:3]):
        torch.testing.assert_close(b, a, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(outs[1][3].float(), outs[0][3].float(), rtol=8e-3, atol=1e-6)


def test_split_key_attention_kernels_match_fp32():
    """Ring-attention building blocks on the GPU: per-source partial forwards (keys split over three
    sources, as context-parallel ranks hold them), the log-sum-exp merge kernel, and the per-source
    backward against the final (o, lse) with dQ accumulated in fp32, against fp32 autograd."""
    from axrl_b200.ops import core as ops
    from axrl_b200.ops.attention_spec import spec_from_triples

    torch.manual_seed(11)
    T, Hq, Hkv, D = 384, 8, 2, 128
    bounds = [(0, 256), (256, 512), (512, 768)]
    # local queries: rows 0-191 see all of source 0 and a causal diagonal in source 1; rows 192-383
    # see source 2 fully and nothing of source 0 (an empty partial the merge must skip)
    triples = [(0, 192, 0, 256, 0), (0, 192, 256, 448, 1), (192, 384, 512, 768, 0), (192, 384, 448, 512, 0)]
    scale = D ** -0.5
    q = torch.randn(T, Hq, D, device=DEV).bfloat16()
    k = torch.randn(768, Hkv, D, device=DEV).bfloat16()
    v = torch.randn(768, Hkv, D, device=DEV).bfloat16()
    do = torch.randn(T, Hq, D, device=DEV).bfloat16()
    full = spec_from_triples(triples, T, 768)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref = ops._attn_ref(qf, kf, vf, full, scale)
    o_ref.float().backward(do.float())
    srcs = []
    for a, b in bounds:
        tr = []
        for q0, q1, k0, k1, t in triples:
            ka, kb = max(k0, a), min(k1, b)
            qa = q0 + (ka - k0) if t == 1 else q0
            if ka < kb and qa < q1:
                tr.append((qa, q1, ka - a, kb - a, t))
        srcs.append(spec_from_triples(tr, T, b - a).to(DEV))
    parts = [ops.attn_partial(q, k[a:b], v[a:b], sp, scale) for (a, b), sp in zip(bounds, srcs)]
    o, lse2 = ops.attn_merge(parts)
    dsum = ops.attn_bwd_dsum(o, do)
    dq = torch.zeros(T, Hq, D, device=DEV)
    grads = [ops.attn_bwd_partial(do, q, k[a:b], v[a:b], lse2, dsum, dq, sp, scale) for (a, b), sp in zip(bounds, srcs)]
    torch.cuda.synchronize()
    assert _ext().attn_tc_error() == 0 and _ext().attn_bwd_tc_error() == 0
    close(o, o_ref, 2e-2, 1e-2, msg="merged o")
    close(dq, qf.grad, 3e-2, 2e-2, msg="dq")
    close(torch.cat([g[0] for g in grads]), kf.grad, 3e-2, 2e-2, msg="dk")
    close(torch.cat([g[1] for g in grads]), vf.grad, 3e-2, 2e-2, msg="dv")


@pytest.mark.parametrize("k", [1, 8])
def test_moe_combine_matches_index_add(k):
    """Weighted top-k combine of expert rows (one gather per token, fp32 sums) and its backward,
    against the fp32 scatter with index_add and autograd."""
    from axrl_b200.ops.grouped import moe_combine

    torch.manual_seed(k)
    T, H, E = 777, 2048, 64
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)])
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    y = torch.randn(T * k, H, device=DEV).bfloat16().requires_grad_(True)
    w = torch.rand(T, k, device=DEV).requires_grad_(True)
    out = moe_combine(y, w, order)
    g = torch.randn(T, H, device=DEV).bfloat16()
    out.backward(g)
    yr, wr = y.detach().float().requires_grad_(True), w.detach().clone().requires_grad_(True)
    ref = torch.zeros(T, H, device=DEV).index_add_(0, order // k, yr * wr.reshape(-1)[order][:, None])
    ref.backward(g.float())
    close(out, ref, 2e-2, 1e-2, msg="combine")
    close(y.grad, yr.grad, 1e-2, 1e-2, msg="dy")
    close(w.grad, wr.grad, 5e-2, 1e-3, msg="dw")
