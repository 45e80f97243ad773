"""Worker for the expert-parallel tests (run under torchrun or mp.spawn).

Each rank routes its own tokens through an EP MoE layer holding only its
experts, and checks the result against the unsharded MoE computed locally."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run(rank, world, impl, port, device_kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from mod_b200.config import get_preset
    from mod_b200.models.backend import make_backend
    from mod_b200.models.weights import random_weights
    from mod_b200.parallel import dist as mdist
    from mod_b200.parallel.ep import FusedEPMoE, NcclEPMoE

    mdist.init(backend="gloo" if device_kind == "cpu" else "nccl")
    dev = torch.device("cpu") if device_kind == "cpu" else torch.device("cuda", rank)
    dtype = torch.float32 if device_kind == "cpu" else torch.bfloat16
    cfg = get_preset("tiny-moe")
    cfg.num_hidden_layers = 1
    El = cfg.num_experts // world
    full = random_weights(cfg, device=dev, dtype=dtype, seed=0)
    shard = random_weights(cfg, device=dev, dtype=dtype, seed=0, expert_range=(rank * El, (rank + 1) * El))
    for w in (full, shard):
        w.layers[0].moe.router.mul_(50.0)
    be = make_backend("torch" if device_kind == "cpu" else "native")
    torch.manual_seed(100 + rank)
    T = 5 + 3 * rank
    x = (torch.randn(T, cfg.hidden_size, device=dev) * 0.5).to(dtype)
    ref = make_backend("torch").moe(x, full.layers[0].moe, cfg.num_experts_per_tok, True, cfg.moe_intermediate_size)
    if impl == "nccl":
        moe = NcclEPMoE(cfg, be)
    elif impl == "agrs":  # NVLS all-gather -> local experts -> in-switch reduce; the P2P path as fallback
        from mod_b200.parallel.ep_agrs import AgRsEPMoE

        moe = AgRsEPMoE(cfg, be, max_tokens=32, fallback=FusedEPMoE(cfg, be, max_tokens=16))
    else:
        moe = FusedEPMoE(cfg, be, max_tokens=16)
    scale = ref.float().abs().max().item()
    assert scale > 0, "reference MoE output is all zeros"
    tol = 1e-4 if dtype == torch.float32 else 3e-2  # relative to the output's magnitude
    modes = [None]
    if impl == "fused":  # separate router / top-k / dispatch launches, then the fused route + dispatch kernel
        modes = [False, True]
    for fused_route in modes:
        if fused_route is not None:
            moe.fused_route = fused_route
        for rep in range(3):  # repeated calls exercise the epoch / buffer reuse
            out = moe(x, shard.layers[0].moe)
            err = (out.float() - ref.float()).abs().max().item()
            assert err < tol * scale, f"rank {rank} rep {rep} fused_route={fused_route}: max err {err} vs scale {scale}"
    if impl in ("fused", "agrs"):
        # combine deferred into the next residual add + RMSNorm
        from mod_b200.ops import reference as R

        nw = (1.0 + 0.1 * torch.randn(cfg.hidden_size, device=dev)).to(dtype)
        for rep in range(4 if impl == "agrs" else 2):
            res = (torch.randn(T, cfg.hidden_size, device=dev) * 0.5).to(dtype)
            res_ref = res.clone()
            want = R.rmsnorm(ref.to(dtype), nw, 1e-6, residual=res_ref)
            got = moe(x, shard.layers[0].moe, defer=True).add_norm(res, nw, 1e-6)
            assert torch.allclose(res.float(), res_ref.float(), rtol=2e-2, atol=2e-2 * res_ref.float().abs().max().item())
            err = (got.float() - want.float()).abs().max().item()
            assert err < 3e-2 * want.float().abs().max().item(), f"rank {rank} deferred combine: max err {err}"
    if device_kind != "cpu":
        from mod_b200.ops import check_status
        torch.cuda.synchronize()
        check_status()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    # torchrun entry: python -m torch.distributed.run --nproc-per-node N tests/_ep_worker.py IMPL
    run(int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), sys.argv[1], int(os.environ["MASTER_PORT"]), "cuda")
