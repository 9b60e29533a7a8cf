"""Context-parallel prefill (s1_model_forward_cp): a prompt split into pieces on 64-token
boundaries, one rank per piece, per-layer GDN states, conv history and attention K/V
passed rank to rank over NCCL. The last rank's logits and final hidden row equal, bit for
bit, those of the whole prompt on one GPU, and are within 2e-2 of the oracle. Each case
is skipped with fewer GPUs than pieces."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("pieces", ["256,192", "64,321", "128,64,192,100"])
def test_context_parallel_equals_one_gpu(pieces):
    """Two ranks (first and last only), and four (middle ranks receive, append and send)."""
    import torch
    world = len(pieces.split(","))
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cp_worker.py")
    env = dict(os.environ, CP_PIECES=pieces, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(world), "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), worker]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    out = json.loads(line)
    assert out["fault"] == 0
    assert out["bit_exact_logits"] and out["bit_exact_hidden"], out
    assert out["max_abs_vs_oracle"] <= 2e-2, out
