"""Worker program for the multi-GPU tests (launched by torch.distributed.run, one rank per GPU)."""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _tiny():
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128)
    m = Qwen3Model(cfg)
    m.init_weights(0)
    return cfg, m.to("cuda", torch.bfloat16)


def case_dist_optim() -> None:
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.parallel.dist_optim import DistributedAdamW
    from axrl_b200.train.optimizer import FlatAdamW

    rank, world = dist.get_rank(), dist.get_world_size()
    wc = MegatronWorkerConfig()
    wc.lr_scheduler.lr_warmup_steps = 0
    wc.lr_scheduler.max_lr = 1e-2
    results = {}
    for impl in ("replicated", "nccl", "p2p"):
        _, m = _tiny()
        opt = FlatAdamW(m, wc.optimizer, wc.lr_scheduler) if impl == "replicated" else DistributedAdamW(m, wc.optimizer, wc.lr_scheduler, backend=impl)
        for step in range(3):
            opt.zero_grad()
            g = torch.Generator(device="cuda").manual_seed(100 * step + rank)
            for p in opt.params:
                p.main_grad.copy_(torch.randn(p.shape, device="cuda", generator=g))
            if impl == "replicated":
                dist.all_reduce(opt.grad)
                norm = opt.step(grad_scale=0.5)
            else:
                norm = opt.step(grad_scale=0.5)
        torch.cuda.synchronize()
        results[impl] = (torch.cat([p.detach().float().reshape(-1) for p in m.parameters()]), float(norm))
    ref, rn = results["replicated"]
    for impl in ("nccl", "p2p"):
        got, gn = results[impl]
        err = (got - ref).abs().max().item()
        assert err < 2e-2, f"{impl}: max param diff {err}"
        assert abs(gn - rn) / rn < 1e-3, f"{impl}: grad norm {gn} vs {rn}"
    print(f"rank {rank}: dist_optim ok", flush=True)


def case_weight_sync() -> None:
    from axrl_b200.sync.plan import qwen3_param_specs
    from axrl_b200.sync.weight_sync import WeightSyncer

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg, m = _tiny()
    specs = qwen3_param_specs(cfg)
    full = {}
    for name, p in m.named_parameters():
        full[name.replace(".weight", "") if name.endswith("layernorm.weight") is False and name.endswith("norm.weight") is False else name] = p.detach()
    from axrl_b200.sync.plan import _slices

    def local(spec, tp, r):
        t = dict(m.named_parameters())[spec.name if spec.name in dict(m.named_parameters()) else spec.name + ".weight"].detach()
        t = t.reshape(-1, t.shape[-1]) if t.dim() > 1 else t.reshape(1, -1)
        parts, row = [], 0
        for sub in spec.subs:
            blk = t[row:row + sub.rows]
            r0, r1, c0, c1 = _slices(sub, tp)[r]
            parts.append(blk[r0:r1, c0:c1])
            row += sub.rows
        return torch.cat(parts, 0)

    for fp8 in (False, True):
        dst_groups = [[(r + 1) % world for r in range(world)]]  # destination TP rank j lives on rank j+1: cross-GPU writes
        ws = WeightSyncer(specs, src_tp=world, src_ranks=list(range(world)), dst_tp=world, dst_groups=dst_groups, fp8=fp8)
        for spec in specs:
            ws.param_view(spec.name, "src").copy_(local(spec, world, rank))
        secs = ws.push()
        torch.cuda.synchronize()
        j = (rank - 1) % world  # destination TP rank held here
        for spec in specs:
            exp = local(spec, world, j).float()
            got = ws.param_view(spec.name, "dst")
            if fp8 and all(s.split != -1 for s in spec.subs) and got.dtype == torch.float8_e4m3fn:
                sc = ws.scale_view(spec.name)
                deq = got.float() * sc.repeat_interleave(128, 0).repeat_interleave(128, 1)[: got.shape[0], : got.shape[1]]
                err = ((deq - exp).abs() / (exp.abs().max() + 1e-6)).max().item()
                assert err < 0.07, f"{spec.name}: fp8 rel err {err}"
            else:
                assert torch.equal(got.float(), exp), spec.name
        print(f"rank {rank}: weight_sync fp8={fp8} ok ({ws.bytes_pushed / 1e6:.1f} MB pushed in {secs * 1e3:.3f} ms)", flush=True)
        # the NCCL-broadcast baseline produces the same destination contents
        snap = {spec.name: ws.param_view(spec.name, "dst").clone() for spec in specs}
        for spec in specs:
            ws.param_view(spec.name, "dst").zero_()
        ws.push_nccl()
        torch.cuda.synchronize()
        for spec in specs:
            assert torch.equal(ws.param_view(spec.name, "dst").view(torch.uint8), snap[spec.name].view(torch.uint8)), spec.name
        print(f"rank {rank}: weight_sync nccl baseline fp8={fp8} ok", flush=True)


def case_tp(backends=("torch", "p2p")) -> None:
    """TP=world with sequence parallelism: NCCL collectives and the overlapped P2P kernels, each
    against the TP=1 model (same weights) on this GPU.  ``p2p_fused``: the P2P communicator with
    the row-parallel forward GEMM fused with its reduce-scatter (one tcgen05 kernel storing tiles
    into the owners' slots)."""
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.ops.attention_spec import spec_from_triples
    from axrl_b200.parallel import tensor_parallel as tpl

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                      num_key_value_heads=4, head_dim=128)
    full = Qwen3Model(cfg)
    full.init_weights(5)
    full = full.to("cuda", torch.bfloat16)
    full.inv_freq = full.inv_freq.float()
    state = {k: v.detach().clone() for k, v in full.named_parameters()}
    T = 512
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    labels = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    labels[::7] = -100
    spec = spec_from_triples([(0, 200, 0, 200, 1), (200, T, 200, T, 1)], T).to("cuda")
    pos = torch.cat([torch.arange(200), torch.arange(T - 200)]).int().cuda()

    def run(model):
        for p in model.parameters():
            p.main_grad = torch.zeros(p.shape, dtype=torch.float32, device="cuda")
            p.grad = None
        h = model(ids, pos, spec)
        lp, ent = model.logprobs(h, labels, entropy=True)
        keep = (labels >= 0).float()
        ((lp * keep).sum() / keep.sum() + 0.05 * (ent * keep).sum() / keep.sum()).backward()
        for p in model.parameters():
            if p.grad is not None:
                p.main_grad += p.grad.float()
                p.grad = None
        return lp.detach(), ent.detach()

    lp_ref, ent_ref = run(full)
    keep = labels >= 0
    for backend in backends:
        os.environ["AXRL_TP_FUSED"] = "1" if backend == "p2p_fused" else "0"
        tp = tpl.TPContext.from_group(dist.group.WORLD, backend="p2p" if backend == "p2p_fused" else backend)
        if backend == "p2p_fused":
            assert tp.comm.fused
        m = Qwen3Model(cfg, tp=tp).to("cuda", torch.bfloat16)
        m.inv_freq = m.inv_freq.float()
        tpl.load_shards_from_full(m, state, tp)
        lp, ent = run(m)
        tpl.allreduce_replicated_grads(m, tp)
        torch.cuda.synchronize()
        if hasattr(tp.comm, "check"):
            tp.comm.check()
        d_lp = (lp - lp_ref)[keep].abs().max().item()
        d_ent = (ent - ent_ref).abs().max().item()
        assert d_lp < 5e-2 and d_ent < 5e-2, f"{backend}: lp diff {d_lp}, entropy diff {d_ent}"
        worst = 0.0
        for n, p in m.named_parameters():
            gr = p.main_grad
            if not getattr(p, "tp_replicated", False):
                parts = [torch.empty_like(gr) for _ in range(world)]
                dist.all_gather(parts, gr.contiguous())
                gr = tpl.unshard_param(n, parts, cfg)
            ref = dict(full.named_parameters())[n].main_grad
            rel = ((gr - ref).norm() / (ref.norm() + 1e-12)).item()
            worst = max(worst, rel)
            assert rel < 3e-2, f"{backend}: grad {n} rel err {rel}"
        print(f"rank {rank}: tp {backend} ok (lp diff {d_lp:.2e}, worst grad rel err {worst:.2e})", flush=True)


def case_tp_fused() -> None:
    case_tp(("p2p_fused",))


def case_tp_timeout() -> None:
    """A P2P TP wait whose peer never signals returns an error status after its bounded wait
    instead of hanging: rank 1 skips the collective; rank 0 must see the timeout."""
    import os as _os

    _os.environ["AXRL_TP_TIMEOUT_S"] = "1"
    from axrl_b200.parallel.tp_overlap import P2PTPComm

    rank = dist.get_rank()
    comm = P2PTPComm(dist.group.WORLD, cap_tokens=256, hidden=128)
    if rank == 0:
        x = torch.ones(64, 128, dtype=torch.bfloat16, device="cuda")
        comm.all_gather_rows(x)
        torch.cuda.synchronize()
        try:
            comm.check()
            raise AssertionError("expected a timeout")
        except RuntimeError as e:
            assert "timed out" in str(e)
    dist.barrier()
    print(f"rank {rank}: tp timeout ok", flush=True)


def case_ep() -> None:
    """EP=world MoE layer stack: NCCL all-to-all and the NVLink dispatch/combine kernels, each against
    the EP=1 model (same weights) on this rank's own tokens; expert gradients summed over ranks."""
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.ops.attention_spec import spec_from_triples
    from axrl_b200.parallel.expert import EPContext, load_ep_shards_from_full

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                      num_key_value_heads=4, head_dim=128, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256)
    full = Qwen3Model(cfg)
    full.init_weights(9)
    full = full.to("cuda", torch.bfloat16)
    full.inv_freq = full.inv_freq.float()
    state = {k: v.detach().clone() for k, v in full.named_parameters()}
    T = 300 + 64 * rank
    g = torch.Generator().manual_seed(50 + rank)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    labels = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    spec = spec_from_triples([(0, T, 0, T, 1)], T).to("cuda")
    pos = torch.arange(T).int().cuda()

    def run(model):
        for p in model.parameters():
            p.main_grad = torch.zeros(p.shape, dtype=torch.float32, device="cuda")
            p.grad = None
        lp, _ = model.logprobs(model(ids, pos, spec), labels)
        lp.mean().backward()
        for p in model.parameters():
            if p.grad is not None:
                p.main_grad += p.grad.float()
                p.grad = None
        return lp.detach()

    lp_ref = run(full)
    fulld = dict(full.named_parameters())
    for backend in ("torch", "p2p"):
        ep = EPContext.from_group(dist.group.WORLD, backend=backend, hidden=cfg.hidden_size, num_experts=cfg.num_experts,
                                  max_rows=2048 * cfg.num_experts_per_tok)
        m = Qwen3Model(cfg, ep=ep).to("cuda", torch.bfloat16)
        m.inv_freq = m.inv_freq.float()
        load_ep_shards_from_full(m, state, ep)
        lp = run(m)
        torch.cuda.synchronize()
        if hasattr(ep.comm, "check"):
            ep.comm.check()
        d = (lp - lp_ref).abs().max().item()
        assert d < 5e-2, f"{backend}: lp diff {d}"
        worst = 0.0
        for n, p in m.named_parameters():
            ref = fulld[n].main_grad
            if getattr(p, "expert_parallel", False):
                ref = ref.clone()
                dist.all_reduce(ref)
                El = p.shape[0]
                ref = ref[rank * El:(rank + 1) * El]
            rel = ((p.main_grad - ref).norm() / (ref.norm() + 1e-12)).item()
            worst = max(worst, rel)
            assert rel < 3e-2, f"{backend}: grad {n} rel err {rel}"
        print(f"rank {rank}: ep {backend} ok (lp diff {d:.2e}, worst grad rel err {worst:.2e})", flush=True)


def case_zero() -> None:
    """Bucketed ZeRO-1 with the reduce-scatter overlapped with backward (NVLink and NCCL) against the
    replicated optimizer: two GRPO steps on different per-rank data, parameters compared."""
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.models.qwen3 import Qwen3Config
    from axrl_b200.train.engine import ParallelCtx, TrainEngine
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer
    from tests.test_pipeline_parallel import _batch

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=4, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128)

    def engine(zero: str):
        wc = MegatronWorkerConfig(max_tokens_per_micro_batch=64, seed=5)
        wc.lr_scheduler.lr_warmup_steps = 0
        wc.lr_scheduler.max_lr = 1e-3
        e = TrainEngine(wc, cfg, "cuda", par=ParallelCtx(dp_group=dist.group.WORLD, dp_size=world, zero_backend=zero))
        if hasattr(e.optim, "buckets"):
            assert len(e.optim.buckets) >= 2
        return e

    b = _batch()
    b = b.select_rows([i for i in range(len(b)) if i % world == rank])
    trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo"))
    results = {}
    for zero in ("off", "nccl", "p2p"):
        e = engine(zero)
        lp = e.compute_logprobs(b)
        bb = b.select_rows(list(range(len(b))))
        bb["old_logprobs"] = lp
        bb["ref_logprobs"] = lp
        norms = [e.train_step(bb, trainer)["grad_norm"] for _ in range(2)]
        torch.cuda.synchronize()
        if hasattr(e.optim, "check"):
            e.optim.check()
        results[zero] = (torch.cat([p.detach().float().reshape(-1) for p in e.model.parameters()]), norms)
        del e
    ref, rn = results["off"]
    for zero in ("nccl", "p2p"):
        got, gn = results[zero]
        d = (got - ref).abs().max().item()
        assert d < 1e-2, f"{zero}: max param diff {d}"
        assert all(abs(a - b_) / max(b_, 1e-6) < 2e-2 for a, b_ in zip(gn, rn)), f"{zero}: norms {gn} vs {rn}"
        print(f"rank {rank}: zero {zero} ok (max param diff {d:.2e})", flush=True)


def case_rollout_tp() -> None:
    """TP=world rollout engine (sharded weights, fused all-reduce + RMSNorm, gathered logits):
    both ranks generate the same tokens, and the rollout log-probs match a TP=1 trainer recompute."""
    from axrl_b200.configs import MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.parallel import tensor_parallel as tpl
    from axrl_b200.rollout.engine import GenRequest, RolloutEngine
    from axrl_b200.train.engine import TrainEngine

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=8,
                      num_key_value_heads=4, head_dim=128)
    full = Qwen3Model(cfg)
    full.init_weights(7)
    full = full.to("cuda", torch.bfloat16)
    full.inv_freq = full.inv_freq.float()
    state = {k: v.detach().clone() for k, v in full.named_parameters()}
    tp = tpl.TPContext.from_group(dist.group.WORLD)
    shard = Qwen3Model(cfg, tp=tp).to("cuda", torch.bfloat16)
    shard.inv_freq = shard.inv_freq.float()
    tpl.load_shards_from_full(shard, state, tp)
    for p in shard.parameters():
        p.requires_grad_(False)
    for use_graph in (False, True):
        eng = RolloutEngine(shard, max_batch=8, kv_tokens=4096, max_context=256, seed=3, use_cuda_graph=use_graph, burst=8,
                            tp_group=dist.group.WORLD, embed_full=state["embed_tokens"])
        g = torch.Generator().manual_seed(0)
        reqs = [GenRequest(rid=f"r{i}", prompt=torch.randint(1, 2048, (30 + 9 * i,), generator=g).tolist(), max_new_tokens=40,
                           temperature=1.0, stop_token_ids=(), seed_stream=i) for i in range(5)]
        res = eng.generate(reqs)
        torch.cuda.synchronize()
        eng.tp.check()
        toks = torch.tensor([t for r in res for t in r.output_ids], device="cuda")
        other = [torch.empty_like(toks) for _ in range(world)]
        dist.all_gather(other, toks)
        assert all(torch.equal(o, toks) for o in other), "TP ranks sampled different tokens"
        samples = [Sample.from_tokens(q.prompt, r.output_ids, rollout_logprobs=r.output_logprobs) for q, r in zip(reqs, res)]
        batch = SampleBatch.from_samples(samples)
        tr = TrainEngine(MegatronWorkerConfig(inference_only=True), cfg, "cuda", model=full)
        lp = tr.compute_logprobs(batch)
        m = batch["loss_mask"]
        diff = (lp - batch["rollout_logprobs"])[m].abs()
        assert diff.mean().item() < 0.03 and diff.max().item() < 0.6, (diff.mean().item(), diff.max().item())
        eng.release_graphs()
        print(f"rank {rank}: rollout_tp graph={use_graph} ok (mean |dlp| {diff.mean().item():.4f})", flush=True)


def case_cp() -> None:
    """CP=world over NCCL: ring attention (K/V chunks passed around the ring while the per-source
    attention kernels run; dK/dV reduce-scattered around the ring in the backward) and the
    all-gathered path, each against CP=1 on this GPU with the same weights and batch."""
    from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.models.qwen3 import Qwen3Config
    from axrl_b200.train.engine import ParallelCtx, TrainEngine
    from axrl_b200.trainer.grpo_trainer import GrpoTrainer

    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                      num_key_value_heads=4, head_dim=128)
    g = torch.Generator().manual_seed(1)
    samples = []
    for i in range(4):
        p = torch.randint(1, 1024, (300 + 100 * i,), generator=g).tolist()
        r = torch.randint(1, 1024, (200 + 50 * i,), generator=g).tolist()
        samples.append(Sample.from_tokens(p, r, advantage=float(i % 3) - 1.0, rollout_logprobs=(-torch.rand(len(r), generator=g)).tolist(),
                                          trajectory_id=i))
    batch = SampleBatch.from_samples(samples)

    def wc():
        c = MegatronWorkerConfig(max_tokens_per_micro_batch=4096, seed=3)
        c.lr_scheduler.lr_warmup_steps = 0
        c.lr_scheduler.max_lr = 1e-4
        return c

    trainer = GrpoTrainer(GrpoTrainerConfig(loss_type="grpo", loss_agg_type="token-mean"))
    ref = TrainEngine(wc(), cfg, "cuda")
    lp_ref = ref.compute_logprobs(batch)
    batch["old_logprobs"] = lp_ref
    batch["ref_logprobs"] = lp_ref
    gn_ref = ref.train_step(batch, trainer)["grad_norm"]
    mask = batch["loss_mask"].bool()
    for mode in ("ring", "gather"):
        os.environ["AXRL_CP_ATTN"] = mode
        eng = TrainEngine(wc(), cfg, "cuda", par=ParallelCtx(cp_group=dist.group.WORLD, cp_size=world))
        lp = eng.compute_logprobs(batch)
        d = (lp - lp_ref)[mask].abs().max().item()
        gn = eng.train_step(batch, trainer)["grad_norm"]
        torch.cuda.synchronize()
        rel = abs(gn - gn_ref) / max(gn_ref, 1e-6)
        assert d < 5e-2 and rel < 2e-2, f"cp {mode}: lp diff {d}, grad norm {gn} vs {gn_ref}"
        print(f"rank {rank}: cp {mode} ok (lp diff {d:.2e}, grad norm rel {rel:.2e})", flush=True)
    os.environ.pop("AXRL_CP_ATTN", None)


if __name__ == "__main__":
    from datetime import timedelta

    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        globals()[f"case_{sys.argv[1]}"]()
    finally:
        dist.barrier()
        dist.destroy_process_group()
