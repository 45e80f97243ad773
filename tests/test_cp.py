"""Context parallelism on gloo CPU ranks against the unsplit fp32 computation:
ring attention (causal / full, GQA), Ulysses all-to-all attention, and the
gated delta rule with cross-rank state passing."""
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


def _inputs(S, Hq, Hkv, D):
    g = torch.Generator().manual_seed(7)
    return (torch.randn(S, Hq, D, generator=g), torch.randn(S, Hkv, D, generator=g),
            torch.randn(S, Hkv, D, generator=g))


def _worker(rank, world, port, q_out):
    import torch.distributed as dist

    from mod_b200.models.deltanet import chunk_gated_delta_rule
    from mod_b200.ops import reference as R
    from mod_b200.parallel import cp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    errs = {}
    S, Hq, Hkv, D = 24 * world, 8, 4, 32
    q, k, v = _inputs(S, Hq, Hkv, D)
    sl = slice(rank * 24, (rank + 1) * 24)
    for causal in (True, False):
        ref = R.attn_prefill(q, k, v, causal=causal)
        got = cp.ring_attention(q[sl], k[sl], v[sl], causal=causal)
        errs[f"ring_causal{int(causal)}"] = (got - ref[sl]).abs().max().item()
        got = cp.ulysses_attention(q[sl], k[sl], v[sl], causal=causal)
        errs[f"ulysses_causal{int(causal)}"] = (got - ref[sl]).abs().max().item()
    # gated delta rule: 3 chunks of 16 per rank plus a ragged tail, random initial state
    H, L, dk, dv = 2, 40 * world, 16, 16
    gen = torch.Generator().manual_seed(3)
    qq = torch.nn.functional.normalize(torch.randn(H, L, dk, generator=gen), dim=-1)
    kk = torch.nn.functional.normalize(torch.randn(H, L, dk, generator=gen), dim=-1)
    vv = torch.randn(H, L, dv, generator=gen)
    gg = -torch.rand(H, L, generator=gen) * 0.3
    bb = torch.rand(H, L, generator=gen)
    s0 = torch.randn(H, dk, dv, generator=gen) * 0.1
    o_ref, s_ref = chunk_gated_delta_rule(qq, kk, vv, gg, bb, s0.clone(), 16)
    ls = slice(rank * 40, (rank + 1) * 40)
    o, s_end = cp.deltanet_cp(qq[:, ls], kk[:, ls], vv[:, ls], gg[:, ls], bb[:, ls], s0.clone(), 16)
    errs["deltanet_o"] = (o - o_ref[:, ls]).abs().max().item()
    errs["deltanet_state"] = (s_end - s_ref).abs().max().item()
    q_out.put((rank, errs))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_matches_unsplit(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, errs in res.items():
        for name, e in errs.items():
            assert e < 1e-4, (r, name, e)


def test_merge_partials_handles_empty_sides():
    from mod_b200.parallel.cp import attention_with_lse, merge_partials

    q, k, v = _inputs(6, 4, 2, 8)
    o_full, l_full = attention_with_lse(q, k, v, 0.3)
    o1, l1 = attention_with_lse(q, k[:2], v[:2], 0.3)
    o2, l2 = attention_with_lse(q, k[2:], v[2:], 0.3)
    o, l = merge_partials(o1, l1, o2, l2)
    assert torch.allclose(o, o_full, atol=1e-5) and torch.allclose(l, l_full, atol=1e-5)
    empty = torch.full_like(l1, float("-inf"))
    o, l = merge_partials(torch.zeros_like(o1), empty, o1, l1)
    assert torch.allclose(o, o1, atol=1e-6) and torch.allclose(l, l1)


def _engine_worker(rank, world, port, name, mode, q_out):
    import torch.distributed as dist

    from mod_b200.config import get_preset
    from mod_b200.engine import SamplingParams
    from mod_b200.engine.llm_engine import LLMEngine

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = get_preset(name)
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, cfg.vocab_size, (37,), generator=g).tolist()   # 37: the last chunk is padded
    params = SamplingParams(max_new_tokens=6, ignore_eos=True)
    eng = LLMEngine(cfg, backend="torch", device="cpu", max_batch=2, max_model_len=64, seed=0,
                    expert_parallel=False, use_graphs=False)
    got = eng.generate_context_parallel(prompt, params, mode=mode)
    single = LLMEngine(cfg, backend="torch", device="cpu", max_batch=2, max_model_len=64, seed=0,
                       expert_parallel=False, use_graphs=False)
    want = single.generate([prompt], params)[0]
    q_out.put((rank, got, want, eng.scheduler.num_resumed))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name,mode", [("tiny-dense", "ring"), ("tiny-dense", "ulysses"), ("tiny-moe", "ring")])
def test_engine_context_parallel_prefill_then_decode(name, mode):
    """A 37-token prompt prefilled over 2 gloo ranks (ring / Ulysses attention), its KV put
    into the engine's paged pool, then decoded by the engine: the same tokens as the
    single-process engine, with no recomputation of the prompt (one swap-in resume)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_engine_worker, args=(r, world, port, name, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, want, resumed in res:
        assert got == want, (rank, got, want)
        assert resumed == 1
