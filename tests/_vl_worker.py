"""Worker for the tensor-parallel vision-language tests: images encoded
data-parallel, visual rows exchanged into the owners' shards, the TP decoder
must reproduce the single-process VL engine."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

SIZE = 64


def run(rank, world, backend, port, device_kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from mod_b200.config import get_preset
    from mod_b200.engine import SamplingParams
    from mod_b200.engine.llm_engine import LLMEngine
    from mod_b200.models.backend import make_backend
    from mod_b200.models.tp_decoder import shard_weights
    from mod_b200.models.vl import TPVLModel, VLModel, random_vl_weights
    from mod_b200.parallel import dist as mdist
    from mod_b200.parallel.tp import FusedTP, FusedVisionExchange, NcclTP, NcclVisionExchange

    mdist.init(backend="gloo" if device_kind == "cpu" else "nccl")
    dev = torch.device("cpu") if device_kind == "cpu" else torch.device("cuda", rank)
    dtype = torch.float32 if device_kind == "cpu" else torch.bfloat16
    cfg = get_preset("tiny-vl")
    cfg.text.num_attention_heads, cfg.text.num_key_value_heads = 8, 4
    be = make_backend(backend)
    tw, vw = random_vl_weights(cfg, device=dev, dtype=dtype, seed=0)
    g = torch.Generator().manual_seed(5)
    imgs = [torch.rand(3, SIZE, SIZE, generator=g) for _ in range(3)]
    texts = [torch.randint(0, 400, (n,), generator=g).tolist() for n in (3, 6, 2, 5)]
    params = SamplingParams(max_new_tokens=5, ignore_eos=True)

    def serve(eng, model):
        ids = []
        for k, t in enumerate(texts):  # three image prompts and one text-only prompt
            if k < 3:
                ids.append(eng.add_request(model.prompt_with_image(t), params, images=imgs[k].to(dev, dtype)))
            else:
                ids.append(eng.add_request(t, params))
        while eng.has_unfinished():
            eng.step()
        return [eng.seqs[i].output for i in ids]

    H = cfg.text.hidden_size
    if backend == "native":
        comm, vx = FusedTP(H, 256), FusedVisionExchange(H, 256)
    else:
        comm, vx = NcclTP(H, 256), NcclVisionExchange(be)
    tp_model = TPVLModel(cfg, shard_weights(cfg.text, tw, rank, world), vw, be, comm, world, vx, image_size=SIZE)
    tp = LLMEngine(cfg.text, model=tp_model, backend=backend, device=dev, max_batch=4, max_model_len=64,
                   tensor_parallel=True, use_graphs=False)
    out = serve(tp, tp_model)
    tw1, vw1 = random_vl_weights(cfg, device=dev, dtype=dtype, seed=0)
    single_model = VLModel(cfg, tw1, vw1, make_backend(backend), image_size=SIZE)
    single = LLMEngine(cfg.text, model=single_model, backend=backend, device=dev, max_batch=4, max_model_len=64,
                       expert_parallel=False, use_graphs=False)
    ref = serve(single, single_model)
    if device_kind == "cpu":
        assert out == ref, (out, ref)
    else:
        agree = sum(a == b for x, y in zip(out, ref) for a, b in zip(x, y)) / sum(len(x) for x in ref)
        assert all(x[0] == y[0] for x, y in zip(out, ref)) and agree >= 0.8, (out, ref)
        from mod_b200.ops import check_status

        torch.cuda.synchronize()
        check_status()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    run(int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), sys.argv[1], int(os.environ["MASTER_PORT"]), "cuda")
