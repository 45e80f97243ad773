"""Tensor-parallel vision-language: data-parallel vision encoder, visual rows
delivered to the owners of their token rows, TP decoder."""
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn_cpu(rank, world, port):
    sys.path.insert(0, HERE)
    import _vl_worker

    _vl_worker.run(rank, world, "torch", port, "cpu")


@pytest.mark.parametrize("world", [2])
def test_vl_tp_gloo_matches_single(world):
    mp.spawn(_spawn_cpu, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.gpu
def test_vl_tp_fused_exchange_multi_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_vl_worker.py"), "native"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
