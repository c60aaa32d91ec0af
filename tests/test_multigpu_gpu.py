"""Multi-GPU parity of the fused backward + cross-GPU dB / dC sum
(ssm_bwd_bc_multicast through parallel.MulticastBCSum).  Needs two GPUs on one
node; skipped with fewer.  The ranks run as a torch.distributed.run child."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_channel_shards_sum_bc_through_multicast():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(min(n, 4)),
           "--master-addr", "127.0.0.1", "--master-port", "29631", os.path.join(ROOT, "tests", "_bc_multicast_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=540, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("{")][-1]
    res = json.loads(line)
    if "skip" in res:
        pytest.skip(res["skip"])
    assert res["f32"]["worst"] < 1e-5, res["f32"]
    # bf16 outputs: the same fp32 sums rounded once; allow a couple of bf16 ulps
    assert res["bf16"]["worst"] < 2e-2, res["bf16"]
