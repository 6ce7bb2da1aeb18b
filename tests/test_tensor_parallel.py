"""Tensor + sequence parallelism on CPU: two gloo ranks (TP=2) against one TP=1 model.

Checks the column/row-parallel blocks, vocabulary-parallel embedding and log-prob/entropy,
the replicated-gradient all-reduce and the shard/unshard helpers (cf. the reference's reliance on
Megatron TP+SP, ``axrl/worker/megatron_worker.py:825``)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(moe: bool | str = False):
    """``moe``: False (dense), True (MoE) or "hybrid" (Qwen3.5 style: Gated DeltaNet + gated attention
    with partial RoPE, MoE with a shared expert)."""
    from axrl_b200.models.qwen3 import Qwen3Config

    kw = dict(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16)
    if moe:
        kw.update(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32)
    if moe == "hybrid":
        kw.update(layer_types=["linear_attention", "full_attention"], linear_num_key_heads=2, linear_num_value_heads=4,
                  linear_key_head_dim=16, linear_value_head_dim=8, attn_output_gate=True, partial_rotary_factor=0.5,
                  zero_centered_norm=True, shared_expert_intermediate_size=24)
    return Qwen3Config(**kw)


def _batch(T: int, V: int, seed: int = 0):
    from axrl_b200.ops.attention_spec import spec_from_triples

    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, V, (T,), generator=g)
    labels = torch.randint(0, V, (T,), generator=g)
    labels[::5] = -100
    a = T // 3
    spec = spec_from_triples([(0, a, 0, a, 1), (a, T, a, T, 1)], T)
    pos = torch.cat([torch.arange(a), torch.arange(T - a)]).int()
    return ids, pos, spec, labels


def _loss(model, ids, pos, spec, labels):
    h = model(ids, pos, spec)
    lp, ent = model.logprobs(h, labels, temperature=0.9, entropy=True)
    w = (labels >= 0).float()
    return (lp * w).sum() / w.sum() + 0.1 * (ent * w).sum() / w.sum(), lp, ent


def _attach_grads(model):
    for p in model.parameters():
        p.main_grad = torch.zeros(p.shape, dtype=torch.float32)


def _worker(rank: int, world: int, port: int, moe: bool, q) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from axrl_b200.models.qwen3 import Qwen3Model
        from axrl_b200.parallel import tensor_parallel as tpl

        cfg = _cfg(moe)
        torch.manual_seed(0)
        full = Qwen3Model(cfg)
        full.init_weights(3)
        full_state = {k: v.detach().clone() for k, v in full.named_parameters()}
        tp = tpl.TPContext.from_group(dist.group.WORLD)
        model = Qwen3Model(cfg, tp=tp)
        tpl.load_shards_from_full(model, full_state, tp)
        ids, pos, spec, labels = _batch(24, cfg.vocab_size)

        _attach_grads(full)
        loss_ref, lp_ref, ent_ref = _loss(full, ids, pos, spec, labels)
        loss_ref.backward()
        _attach_grads(model)
        loss, lp, ent = _loss(model, ids, pos, spec, labels)
        loss.backward()
        for m in (full, model):  # autograd .grad (CPU ops) folded into main_grad, as the optimizer does
            for p in m.parameters():
                if p.grad is not None:
                    p.main_grad += p.grad.float()
                    p.grad = None
        tpl.allreduce_replicated_grads(model, tp)

        keep = labels >= 0  # ignored rows carry no defined log-prob
        torch.testing.assert_close(lp[keep], lp_ref[keep], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(ent, ent_ref, atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(loss, loss_ref, atol=1e-5, rtol=1e-5)

        def grads(m):
            out = {}
            for n, p in m.named_parameters():
                g = p.main_grad.clone()
                if p.grad is not None:
                    g += p.grad.float()
                out[n] = g
            return out

        g_tp = grads(model)
        g_ref = grads(full)
        for n, p in model.named_parameters():
            if getattr(p, "tp_replicated", False):
                got = g_tp[n]
            else:
                parts = [torch.empty_like(g_tp[n]) for _ in range(world)]
                dist.all_gather(parts, g_tp[n].contiguous())
                got = tpl.unshard_param(n, parts, cfg)
            torch.testing.assert_close(got, g_ref[n], atol=2e-4, rtol=2e-3, msg=lambda m, n=n: f"{n}: {m}")
        # gather_full_state round-trips the shards
        st = tpl.gather_full_state(model, tp)
        for n in full_state:
            torch.testing.assert_close(st[n], full_state[n])
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
        raise e
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("moe", [False, True, "hybrid"])
def test_tp2_matches_tp1(moe):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, moe, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"


@pytest.mark.parametrize("kind", [False, "hybrid"])
def test_shard_unshard_roundtrip(kind):
    from axrl_b200.models.qwen3 import Qwen3Model
    from axrl_b200.parallel import tensor_parallel as tpl

    cfg = _cfg(kind)
    m = Qwen3Model(cfg)
    m.init_weights(1)
    for n, p in m.named_parameters():
        for tp in (2, 4):
            if p.dim() >= 2 and n.endswith("qkv_proj") and cfg.num_key_value_heads % tp:
                continue
            if cfg.linear_num_key_heads % tp and n.startswith("layers.0.self_attn."):  # GDN layer 0: 2 key heads
                continue
            shards = [tpl.shard_param(n, p.detach(), r, tp, cfg) for r in range(tp)]
            torch.testing.assert_close(tpl.unshard_param(n, shards, cfg), p.detach())


def test_pack_rows_pad_to():
    from axrl_b200.data.sample import Sample, SampleBatch
    from axrl_b200.train.packing import pack_rows

    samples = [Sample.from_tokens(list(range(1, 6)), [7, 8, 9]), Sample.from_tokens(list(range(2, 9)), [3])]
    b = SampleBatch.from_samples(samples)
    mb = pack_rows(b, [0, 1], pad_to=16)
    assert mb.num_tokens == 16 and mb.spec.total_q == 16
    assert (mb.labels[sum(mb.row_len):] < 0).all() and not mb.loss_mask[sum(mb.row_len):].any()
    dense = mb.unpack(torch.arange(16).float(), b["input_ids"].shape[1])
    assert dense.shape == (2, b["input_ids"].shape[1])
    assert dense[1, 0].item() == mb.row_off[1]
