"""Engine server + router launched as processes (tiny model on CPU), and placement arithmetic
(reference ``axrl/utils/sglang_launch_utils.py``, ``axrl/pipeline/utils.py:242-348``)."""

import pytest
import requests

from axrl_b200.pipeline.placement import get_worker_placement


def test_placement():
    p = get_worker_placement(8, colocated=True, rollout_tp=2, trainer_model_parallel=2, with_value=True)
    assert p.trainer_ranks == list(range(8)) and p.rollout_engines == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert p.roles_of(3) == ["trainer", "rollout", "value"]
    d = get_worker_placement(8, colocated=False, trainer_gpus=4, rollout_tp=2)
    assert d.trainer_ranks == [0, 1, 2, 3] and d.rollout_engines == [[4, 5], [6, 7]] and d.roles_of(5) == ["rollout"]
    with pytest.raises(AssertionError):
        get_worker_placement(8, colocated=False, trainer_gpus=3, rollout_tp=2)


@pytest.mark.timeout(300)
def test_launch_two_servers_and_router():
    from axrl_b200.serve.launch import launch_servers

    g = launch_servers("tiny", ["cpu", "cpu"], extra_args=["--max-batch", "4", "--max-context", "256"], timeout_s=240)
    try:
        for i in range(3):
            r = requests.post(g.router_url + "/generate", json={"rid": f"s{i % 2}", "input_ids": list(range(5, 25)),
                                                               "sampling_params": {"max_new_tokens": 6, "temperature": 1.0}}, timeout=120)
            r.raise_for_status()
            out = r.json()
            assert len(out["output_ids"]) == 6 and len(out["meta_info"]["output_token_logprobs"]) == 6
        assert requests.get(g.router_url + "/health", timeout=5).json()["backends"] == 2
    finally:
        g.stop()
