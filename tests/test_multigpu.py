"""Multi-GPU paths (run only with >= 2 GPUs): distributed optimizer (NCCL and fused P2P) against a
replicated reference, and the weight-sync push kernel (bf16 and block-fp8) across GPUs."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
HERE = os.path.dirname(os.path.abspath(__file__))


def _run(case: str, n: int = 2) -> str:
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}", "--master-addr=127.0.0.1",
           "--master-port=29533", os.path.join(HERE, "multigpu_worker.py"), case]
    env = dict(os.environ, NCCL_DEBUG="WARN")
    p = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return p.stdout


def test_dist_optim_two_gpus():
    assert _run("dist_optim").count("dist_optim ok") == 2


def test_weight_sync_two_gpus():
    out = _run("weight_sync")
    assert out.count("weight_sync fp8") == 4 and out.count("nccl baseline") == 4, out[-2000:]


def test_tensor_parallel_two_gpus():
    out = _run("tp")
    assert out.count("tp torch ok") == 2 and out.count("tp p2p ok") == 2, out[-2000:]


def test_tensor_parallel_fused_gemm_rs_two_gpus():
    """Row-parallel forward GEMM fused with its reduce-scatter (tcgen05 tiles stored into peer slots)."""
    out = _run("tp_fused")
    assert out.count("tp p2p_fused ok") == 2, out[-2000:]


def test_tp_p2p_wait_times_out_without_hanging():
    assert _run("tp_timeout").count("tp timeout ok") == 2


def test_expert_parallel_two_gpus():
    out = _run("ep")
    assert out.count("ep torch ok") == 2 and out.count("ep p2p ok") == 2, out[-2000:]


def test_context_parallel_ring_two_gpus():
    out = _run("cp")
    assert out.count("cp ring ok") == 2 and out.count("cp gather ok") == 2, out[-2000:]


def test_bucketed_zero_two_gpus():
    out = _run("zero")
    assert out.count("zero nccl ok") == 2 and out.count("zero p2p ok") == 2, out[-2000:]


def test_tensor_parallel_rollout_two_gpus():
    out = _run("rollout_tp")
    assert out.count("rollout_tp graph=False ok") == 2 and out.count("rollout_tp graph=True ok") == 2, out[-2000:]
