"""Worker for tensor-parallel tests: the TP engine (sequence-parallel, NCCL/gloo
or fused NVLink boundaries) must reproduce the single-process engine."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run(rank, world, backend, port, device_kind, preset="tiny-dense"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from mod_b200.config import get_preset
    from mod_b200.engine import SamplingParams
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.weights import random_weights
    from mod_b200.parallel import dist as mdist

    mdist.init(backend="gloo" if device_kind == "cpu" else "nccl")
    dev = torch.device("cpu") if device_kind == "cpu" else torch.device("cuda", rank)
    dtype = torch.float32 if device_kind == "cpu" else torch.bfloat16
    cfg = get_preset(preset)
    if preset == "tiny-dense":
        cfg.num_attention_heads, cfg.num_key_value_heads = max(8, 2 * world), max(4, world)  # heads divide the ranks
    w = random_weights(cfg, device=dev, dtype=dtype, seed=0)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 19, 3)]
    params = SamplingParams(max_new_tokens=6)
    tp = LLMEngine(cfg, weights=w, backend=backend, device=dev, max_batch=4, max_model_len=64, tensor_parallel=True)
    out = tp.generate(prompts, params)
    w1 = random_weights(cfg, device=dev, dtype=dtype, seed=0)
    single = LLMEngine(cfg, weights=w1, backend=backend, device=dev, max_batch=4, max_model_len=64,
                       expert_parallel=False, use_graphs=False)
    ref = single.generate(prompts, params)
    if device_kind == "cpu":
        assert out == ref, (out, ref)
        # the same TP engine built from an HF checkpoint: each rank maps only its own slices
        import tempfile

        from mod_b200.io.safetensors import save_file
        from tests.test_io import _hf_from_fused

        with tempfile.TemporaryDirectory() as d:
            save_file(os.path.join(d, "model.safetensors"), _hf_from_fused(cfg, w1), {})
            ck = LLMEngine(cfg, backend=backend, device=dev, max_batch=4, max_model_len=64, tensor_parallel=True,
                           model_path=d)
            out2 = ck.generate(prompts, params)
        assert out2 == ref, (out2, ref)
    else:  # bf16: the first tokens must agree, the rest mostly
        agree = sum(a == b for x, y in zip(out, ref) for a, b in zip(x, y)) / sum(len(x) for x in ref)
        assert all(x[0] == y[0] for x, y in zip(out, ref)) and agree >= 0.8, (out, ref)
        from mod_b200.ops import check_status
        torch.cuda.synchronize()
        check_status()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    run(int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), sys.argv[1], int(os.environ["MASTER_PORT"]), "cuda",
        sys.argv[2] if len(sys.argv) > 2 else "tiny-dense")
