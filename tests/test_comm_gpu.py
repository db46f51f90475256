"""GPU: the NCCL C ABI (`libhb_comm.so`). Failure detection without a GPU fault: a communicator whose second
rank never joins ends in HB_ERR_TIMEOUT at the host-side deadline (one GPU). On two GPUs: the band halo
exchange and the uneven head-pair all-gather through the C ABI, checked exactly."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_comm_init_times_out_when_a_rank_never_joins(cuda_lib):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run([sys.executable, os.path.join(HERE, "_comm_timeout_worker.py")], capture_output=True,
                         text=True, timeout=120, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_comm_halo_exchange_and_pair_gather_two_gpus(cuda_lib):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_comm_two_gpu_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
