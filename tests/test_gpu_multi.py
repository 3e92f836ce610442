"""Multi-GPU sequence sharding with the real NCCL all-gather: two (or more) ranks launched with
torchrun on the GPUs of this box.  Skipped on a box with a single GPU (the one-GPU emulation in
test_gpu_seqshard.py and the gloo test cover the same path there)."""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from tests._helpers import BF16_MAX_ABS, BF16_MIN_COS

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "p2p", "ce"])
def test_seq_shard_two_gpus(tmp_path, mode):
    """The k'|v' exchange by NCCL all-gather, by the prologue's NVLink stores into the peer's buffer
    (CUDA IPC mapping), and by copy-engine pushes into it."""
    out = tmp_path / "outcome.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "_seqshard_worker.py"), str(out), mode]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(out.read_text())
    assert res["world"] == 2 and res["mode"] == mode
    assert res["equal_to_fused"], res
    assert res["max_abs_vs_oracle"] <= BF16_MAX_ABS and res["min_cos_vs_oracle"] >= BF16_MIN_COS, res
