"""GPU (2 GPUs; skipped on fewer): one clip's denoise step split over two ranks equals one GPU's step, both
ways the DiT splits: one batch row per rank (no collective inside the step), and token rows for the token-wise
ops with head pairs for the fused self-attention kernel (NCCL all-to-alls)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("split_batch", ["1", "0"])
def test_dit_step_split_over_two_gpus_matches_one(cuda_lib, split_batch):
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(here, "_dit_two_gpu_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", HB_DIT_SPLIT_BATCH=split_batch)
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
