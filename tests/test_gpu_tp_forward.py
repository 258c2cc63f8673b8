"""Tensor-parallel integer forward on 2+ GPUs (peer memory): greedy tokens and
logits equal the unsharded single-GPU model and the CPU oracle bit for bit
(tests/tp_forward_worker.py, one process per GPU). Skipped on boxes with fewer
than two GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_forward_bit_identical(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "verdict.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "tp_forward_worker.py"), "--out", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    verdict = json.loads(out.read_text())
    for k, v in verdict.items():
        if k != "world":
            assert v["all_ranks"], (k, v)
