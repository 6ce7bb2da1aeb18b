"""Utilities: resource monitor, distributed layout, networking, compressed pickles, session
timeline, and the flat-vs-merged per-layer diff (reference ``axrl/utils/*``)."""

import json
import time

import torch


def test_resource_monitor_samples():
    from axrl_b200.utils.system_monitor import ResourceMonitor, host_metrics, process_metrics

    assert process_metrics()["system/process_open_fds"] > 0
    assert 0 <= host_metrics()["system/mem_used_frac"] <= 1
    got = []
    mon = ResourceMonitor(got.append, interval_s=0.05, gpu=False).start()
    time.sleep(0.3)
    mon.stop()
    assert len(got) >= 2 and "system/load_1m" in got[0]


def test_dist_layout_roundtrip():
    from axrl_b200.utils.dist_utils import DistLayout

    L = DistLayout(tp=2, cp=1, dp=2, pp=2)
    assert L.world == 8
    for r in range(8):
        assert L.rank_of(**L.coords(r)) == r
    assert sorted(L.group_ranks("tp")) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert [0, 4] in L.group_ranks("pp")
    assert sorted(sum(L.group_ranks("dp"), [])) == list(range(8))


def test_network_helpers():
    from axrl_b200.utils.network_utils import get_free_port, get_local_ip, is_port_free

    p = get_free_port()
    assert is_port_free(p) and get_local_ip()


def test_zst_roundtrip(tmp_path):
    from axrl_b200.utils.zst_utils import load_zst, save_zst

    obj = {"a": torch.arange(10), "b": [1, "x"]}
    p = save_zst(obj, tmp_path / "x.zst")
    back = load_zst(p)
    assert torch.equal(back["a"], obj["a"]) and back["b"] == obj["b"]


def test_session_timeline(tmp_path, monkeypatch):
    from axrl_b200.utils.timer import SessionTimer
    from axrl_b200.utils.visualize_session_timer import load_spans, render

    path = tmp_path / "tl.jsonl"
    monkeypatch.setenv("AXRL_SESSION_TIMELINE", str(path))
    for s in ("s1", "s2"):
        with SessionTimer(s, "generate", "rollout"):
            time.sleep(0.01)
        with SessionTimer(s, "tool", "search"):
            pass
    spans = load_spans(path)
    assert len(spans) == 4 and all(sp["end"] >= sp["start"] for sp in spans)
    html = render(spans)
    assert html.count("<rect") >= 4 and "generate" in html
    json.dumps(spans)


def test_prefix_merging_layer_diff_is_tiny_in_fp32():
    from axrl_b200.data.prefix_tree import merge_trajectory_samples
    from axrl_b200.data.sample import Sample
    from axrl_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from axrl_b200.utils.layer_diff import prefix_merging_layer_diff

    cfg = Qwen3Config(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16)
    m = Qwen3Model(cfg)
    m.init_weights(2)
    prompt = list(range(3, 20))
    turns = [Sample.from_tokens(prompt, [40 + i, 41 + i, 42]) for i in range(3)]
    merged = merge_trajectory_samples(turns, align_size=1)
    rows = prefix_merging_layer_diff(m, [list(s.input_ids) for s in turns], merged)
    assert len(rows) == cfg.num_hidden_layers + 1
    assert all(r["max_abs"] < 1e-4 * max(1.0, r["ref_mean_abs"]) for r in rows), rows


def test_tunnel_waits_for_url_and_stops(tmp_path):
    import asyncio
    import sys

    import pytest

    from axrl_b200.utils.tunnel import Tunnel, TunnelConfig

    script = tmp_path / "fake_tunnel.py"
    script.write_text("import sys, time\nprint('starting', flush=True)\nprint('ready at https://abc-def.trycloudflare.com/ port', sys.argv[1], flush=True)\n"
                      "time.sleep(60)\n")

    async def go():
        cfg = TunnelConfig(command=[sys.executable, str(script), "{port}"], startup_timeout_seconds=20)
        t = await Tunnel.start(cfg, template_vars={"port": 8123})
        assert t.base_url == "https://abc-def.trycloudflare.com"
        assert any("8123" in ln for ln in t.lines)
        await t.stop()
        assert t.process.returncode is not None
        bad = TunnelConfig(command=[sys.executable, "-c", "print('no url here')"], startup_timeout_seconds=20)
        with pytest.raises(RuntimeError, match="exited before"):
            await Tunnel.start(bad, template_vars={})
        with pytest.raises(FileNotFoundError):
            await Tunnel.start(TunnelConfig(command=["definitely-not-a-binary-xyz"]), template_vars={})

    asyncio.run(go())


def test_hf_download_skips_existing_and_reports_offline(tmp_path, monkeypatch):
    import pytest

    from axrl_b200.configs import HfDataConfig
    from axrl_b200.utils import hf_download

    cfg = HfDataConfig(repo_id="org/ds", filename="x.parquet")
    monkeypatch.setattr(HfDataConfig, "get_full_path", lambda self: tmp_path / "org" / "ds" / "x.parquet")
    (tmp_path / "org" / "ds").mkdir(parents=True)
    (tmp_path / "org" / "ds" / "x.parquet").write_bytes(b"1")
    assert hf_download.download_data_file(cfg) == tmp_path / "org" / "ds" / "x.parquet"

    class Offline:
        def snapshot_download(self, **kw):
            raise OSError("no network")

    monkeypatch.setattr(hf_download, "_hub", lambda: Offline())
    from axrl_b200.configs import ModelConfig

    with pytest.raises(RuntimeError, match="could not download"):
        hf_download.download_model(ModelConfig(name="org/model"))
