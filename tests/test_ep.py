"""Expert-parallel MoE: baseline on gloo CPU ranks, fused path on GPUs."""
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
    import _ep_worker

    _ep_worker.run(rank, world, "nccl", port, "cpu")


@pytest.mark.parametrize("world", [2, 4])
def test_ep_baseline_gloo_matches_unsharded(world):
    mp.spawn(_spawn_cpu, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.gpu
def test_fused_ep_single_gpu_self_exchange(cuda):
    sys.path.insert(0, HERE)
    import _ep_worker
    import torch.distributed as dist

    _ep_worker.run(0, 1, "fused", _port(), "cuda")
    assert not dist.is_initialized()


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["fused", "nccl", "agrs"])
def test_ep_multi_gpu(cuda, impl):
    """agrs: NVLS all-gather -> local experts -> in-switch reduce (needs NVLink multicast)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    if impl == "agrs":
        from mod_b200.ops import load_extension

        if not all(load_extension().multicast_supported(d) for d in range(n)):
            pytest.skip("no NVLink multicast on these devices")
    n = min(n, 8)  # every visible GPU (up to 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_ep_worker.py"), impl]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


def _pipe_worker(rank, world, port):
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from mod_b200.parallel.pipeline import PipelineExecutor, PipelineStage, split_layers

    torch.manual_seed(0)
    ws = [torch.randn(16, 16) * 0.3 for _ in range(6)]
    layers = [(lambda x, w=w: torch.tanh(x @ w)) for w in ws]
    stages = [PipelineStage(s, r) for r, s in enumerate(split_layers(layers, world))]
    x = torch.randn(8, 16)
    out = PipelineExecutor(stages, micro_batches=4).forward(x if rank == 0 else None, shape=(8, 16))
    if rank == world - 1:
        ref = x
        for f in layers:
            ref = f(ref)
        assert torch.allclose(out, ref, atol=1e-6)
    dist.barrier()
    dist.destroy_process_group()


def test_pipeline_gloo_three_stages():
    mp.spawn(_pipe_worker, args=(3, _port()), nprocs=3, join=True)


def _spawn_tp_cpu(rank, world, port):
    sys.path.insert(0, HERE)
    import _tp_worker

    _tp_worker.run(rank, world, "torch", port, "cpu")


@pytest.mark.parametrize("world", [2, 4])
def test_tp_baseline_gloo_matches_single(world):
    mp.spawn(_spawn_tp_cpu, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.gpu
@pytest.mark.parametrize("backend,cluster", [("native", "0"), ("native", "1"), ("torch", "0")])
def test_tp_multi_gpu(cuda, backend, cluster):
    """cluster=1: decode-sized gathered GEMMs (QKV with the RoPE/KV-write epilogue) as cluster
    launches that wait on the shard flags themselves."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    n = min(n, 8)  # every visible GPU (up to 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MB_TP_CLUSTER=cluster, MB_TP_COMM="p2p")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_tp_worker.py"), backend]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
def test_tp_nvls_multi_gpu(cuda):
    """NVLS boundaries (multimem reduce + multicast stores) reproduce the single-process engine."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    from mod_b200.ops import load_extension

    if not all(load_extension().multicast_supported(d) for d in range(n)):
        pytest.skip("no NVLink multicast on these devices")
    n = min(n, 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MB_TP_COMM="nvls")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_tp_worker.py"), "native"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.parametrize("preset", ["tiny-next", "tiny-moe"])
def test_tp_hybrid_multi_gpu(cuda, preset):
    """Tensor-parallel hybrid / MoE model on 2 GPUs (heads split, experts expert-parallel) against the
    single-process engine."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MB_TP_COMM="p2p")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_tp_worker.py"), "native",
           preset]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
