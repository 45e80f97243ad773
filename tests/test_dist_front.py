"""Multi-process serving front-end: rank 0 takes the requests and streams the
tokens, every rank runs the same loop over its part of the model.  Gloo CPU
ranks: a tensor-parallel dense model and an expert-parallel MoE model, each
request's stream against a single-process engine on the same request."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    from mod_b200.api.dist_front import DistributedFrontEnd
    from mod_b200.config import get_preset
    from mod_b200.engine import SamplingParams
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights
    from mod_b200.parallel import dist as mdist

    mdist.init(backend="gloo")
    if mode == "tp":   # fp32 weights given to every rank (and to the single-process engine)
        cfg = get_preset("tiny-dense")
        cfg.num_attention_heads, cfg.num_key_value_heads = 8, 4
        kw = dict(weights=random_weights(cfg, device="cpu", dtype=torch.float32, seed=0), tensor_parallel=True)
    else:              # each EP rank makes its experts from the same seed
        cfg = get_preset("tiny-moe")
        kw = dict(expert_parallel=True)
    eng = LLMEngine(cfg, backend="torch", device="cpu", max_batch=4, max_model_len=64, use_graphs=False, **kw)
    front = DistributedFrontEnd(eng, mode)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 9, 13)]
    params = [SamplingParams(max_new_tokens=n) for n in (4, 7, 3)]
    if rank == 0:
        rids = [front.submit_request(p, sp) for p, sp in zip(prompts, params)]
        got = [list(front.generate_stream(r, timeout=120)) for r in rids]
        front.shutdown(timeout=120)
        assert front.stats["completed"] == 3
        w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=0) if mode == "tp" else None
        single = LLMEngine(cfg, backend="torch", device="cpu", max_batch=4, max_model_len=64, use_graphs=False,
                           weights=w, expert_parallel=False)
        ref = [single.generate([p], sp)[0] for p, sp in zip(prompts, params)]
        assert [len(x) for x in got] == [sp.max_new_tokens for sp in params]
        assert all(x[:2] == y[:2] for x, y in zip(got, ref)), (got, ref)
        assert sum(a == b for x, y in zip(got, ref) for a, b in zip(x, y)) >= 0.9 * sum(len(y) for y in ref)
    else:
        front.run()  # returns when rank 0 shuts down
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["tp", "ep"])
def test_distributed_front_end_streams_match_single_process(mode):
    mp.spawn(_worker, args=(2, _port(), mode), nprocs=2, join=True)
