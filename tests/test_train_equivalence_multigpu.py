"""Training-step equivalence: N ranks with expert parallelism + hybrid ZeRO follow the
same loss curve as one GPU that accumulates gradients over the same global token set.
(2+ GPUs; both EP token transports, and both ZeRO transports.)"""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "_train_equiv_worker.py")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(cmd, out):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", *cmd, "--out", out], capture_output=True, text=True, env=env,
                       timeout=700)
    assert r.returncode == 0, r.stderr[-3000:]
    with open(out) as f:
        return json.load(f)["losses"]


def compare(single, multi, tol=0.02):
    """Per-step relative agreement of the loss curves; the curve must also fall."""
    assert len(single) == len(multi)
    rel = [abs(a - b) / abs(a) for a, b in zip(single, multi, strict=True)]
    assert max(rel) < tol, (single, multi)
    assert single[-1] < single[0] - 0.2, single  # the repeated batch is being learned
    return max(rel)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport,extra", [("p2p", []), ("nccl", []),
                                             ("p2p", ["--zero-transport", "p2p", "--overlap"])])
def test_ep_zero_step_matches_single_gpu(tmp_path, transport, extra):
    n = min(torch.cuda.device_count(), 8)
    single = _run([sys.executable, WORKER, "--mode", "single"], str(tmp_path / "single.json"))
    multi = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                  "--master-addr=127.0.0.1", f"--master-port={_port()}", WORKER, "--mode", "ep", "--transport",
                  transport, *extra], str(tmp_path / f"ep_{transport}_{len(extra)}.json"))
    compare(single, multi)
