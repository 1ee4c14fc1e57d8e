"""The sharded sampler across real GPUs: torchrun, one process per GPU, NCCL all-gather.
Skipped with fewer than two GPUs."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("config,batch", [(4, 64), (3, 16), (2, 32)])
def test_sharded_sampler_over_nccl(tmp_path, config, batch):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    out = tmp_path / "verdict.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), str(ROOT / "tests" / "sharded_worker.py"),
           "--out", str(out), "--config", str(config), "--batch", str(batch)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    v = json.loads(out.read_text())
    print(v["report"], "unresolved:", v["unresolved"], "world:", v["world"])
    assert v["same_on_all_ranks"]
    assert not v["failures"], v["failures"][:5]
