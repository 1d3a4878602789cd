"""GPU, two or more devices: the sharded algorithms under torchrun (one rank per GPU, NCCL) against the oracle."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_sharded_algorithms_two_ranks(cuda):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29517",
           os.path.join(HERE, "multi_gpu_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    line = [l for l in p.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    for r in out["ranks"]:
        assert r["sumsq_rel"] <= 1e-5
        assert r["dot_rel"] <= 1e-12
        assert r["min_ok"] and r["scan_i32_ok"] and r["scan_u64_ok"] and r["heat_ok"] and r["heat_nccl_ok"]
        assert r["nbody_rel"] <= 1e-4
        assert r["sumsq_fused_rel"] <= 1e-5 and r["fused_matches_nccl"] and r["fused_repeat_ok"] and r["fused_max_ok"]
        assert r["peer_scan_ok"]
