"""Tensor parallelism with the NVLink peer-memory transport on real ranks (one process per GPU)."""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_peer_transport_matches_nccl_on_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(HERE, "_tp_p2p_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    assert out.returncode == 0, out.stderr[-3000:]
    r = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    assert r["ranks_identical"], r
    assert r["p2p_vs_nccl_logits"] < 1e-2 and r["p2p_vs_full_logits"] < 3e-2, r
    assert r["p2p_vs_nccl_grad_max_rel"] < 5e-2 and r["n_grads"] > 10, r
