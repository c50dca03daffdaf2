"""Multi-GPU tests: each launches its worker under torchrun on 2 GPUs (skipped with fewer)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _torchrun(script: str, n: int, timeout: int = 300):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, script)]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout + 60)


def test_expert_parallel_moe_matches_single_gpu_on_two_ranks():
    r = _torchrun("tests/ep_worker.py", 2)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("rel_err") == 2


def test_fused_zero_optimizer_matches_nccl_sharded_adamw_on_two_ranks():
    r = _torchrun("tests/zero_worker.py", 2)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("\"ms_fused\":") == 2


def test_replica_guard_detects_cross_rank_mismatch_on_two_ranks():
    r = _torchrun("tests/guard_worker.py", 2)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count('"mismatch_raised": true') == 2


def test_row_sharded_ple_lookup_over_peer_memory_on_two_ranks():
    r = _torchrun("tests/ple_worker.py", 2)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("peer_vs_contract") == 2
