"""Multi-GPU split-KV decode on real GPUs (skipped with fewer than two): the
in-kernel peer exchange and the NCCL path, two ranks launched as processes."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_peer_split_kv_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mgpu_split_worker.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), worker]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    assert r.stdout.count(" ok") == 2, r.stdout
