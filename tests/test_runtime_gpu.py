"""Engine features on the GPU: sampling, weight streaming, KV swap."""
import pytest
import torch

from mod_b200.config import get_preset
from mod_b200.engine import SamplingParams
from mod_b200.engine.llm_engine import LLMEngine
from mod_b200.models.weights import random_weights

pytestmark = pytest.mark.gpu


def test_weight_streaming_matches_resident(cuda):
    from mod_b200.runtime.offload import enable_streaming

    cfg = get_preset("tiny-dense")
    cfg.num_hidden_layers = 4
    w = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    prompts = [[1, 2, 3, 4, 5], [9, 8, 7]]
    ref = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=2, max_model_len=64,
                    use_graphs=False).generate(prompts, SamplingParams(max_new_tokens=5))
    w2 = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    eng = LLMEngine(cfg, weights=w2, backend="native", device=cuda, max_batch=2, max_model_len=64, use_graphs=False)
    st = enable_streaming(eng.model, resident_layers=1)
    assert not w2.layers[3].attn.qkv.is_cuda
    assert eng.generate(prompts, SamplingParams(max_new_tokens=5)) == ref


def test_sampling_on_gpu_is_seeded(cuda):
    cfg = get_preset("tiny-moe")
    w = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    outs = []
    for _ in range(2):
        eng = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=2, max_model_len=64)
        outs.append(eng.generate([[1, 2, 3]], SamplingParams(max_new_tokens=6, temperature=0.8, top_p=0.9, seed=11)))
    assert outs[0] == outs[1]


def test_kv_swap_roundtrip_gpu(cuda):
    from mod_b200.engine.kv_cache import KVCache
    from mod_b200.runtime.memory import KVSwapper

    kv = KVCache(get_preset("tiny-dense"), 16, cuda)
    for t in kv.k + kv.v:
        t.normal_()
    before = [t[[3, 4]].clone() for t in kv.k + kv.v]
    sw = KVSwapper(kv)
    sw.swap_out(7, [3, 4])
    for t in kv.k + kv.v:
        t.zero_()
    sw.swap_in(7, [10, 11])
    assert all(torch.equal(t[[10, 11]], b) for t, b in zip(kv.k + kv.v, before))


def test_engine_offload_switch_generates_like_resident(cuda):
    """The engine's ``offload_layers`` switch (runtime config / CLI --offload-layers) streams the
    trailing layers from pinned host memory and generates the same tokens."""
    cfg = get_preset("tiny-dense")
    cfg.num_hidden_layers = 4
    prompts = [[1, 2, 3, 4, 5], [9, 8, 7]]
    w = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    ref = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=2, max_model_len=64,
                    use_graphs=False).generate(prompts, SamplingParams(max_new_tokens=5))
    w2 = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    eng = LLMEngine(cfg, weights=w2, backend="native", device=cuda, max_batch=2, max_model_len=64,
                    offload_layers=2)
    assert eng.streamer is not None and not w2.layers[3].attn.qkv.is_cuda and w2.layers[1].attn.qkv.is_cuda
    assert eng.generate(prompts, SamplingParams(max_new_tokens=5)) == ref


def test_preemption_swaps_kv_on_gpu(cuda):
    """Native engine with decode graphs and a KV pool too small for every sequence: preempted
    sequences resume from swapped KV, and the first generated tokens match an unpreempted run."""
    cfg = get_preset("tiny-dense")
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (30, 17, 25, 9)]
    params = SamplingParams(max_new_tokens=40, ignore_eos=True)
    w = random_weights(cfg, device=cuda, dtype=torch.bfloat16, seed=0)
    ref = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=4, max_model_len=96,
                    num_blocks=64).generate(prompts, params)
    eng = LLMEngine(cfg, weights=w, backend="native", device=cuda, max_batch=4, max_model_len=96, num_blocks=14)
    out = eng.generate(prompts, params)
    st = eng.stats()
    assert st["preempted"] > 0 and st["resumed"] == st["swapped_out"] == st["preempted"]
    agree = sum(a == b for x, y in zip(out, ref) for a, b in zip(x, y)) / sum(len(x) for x in ref)
    assert all(x[:4] == y[:4] for x, y in zip(out, ref)) and agree >= 0.9, (out, ref)


def test_staged_upload_and_hf_load_on_gpu(cuda, tmp_path):
    """Pinned double-buffered upload: many small chunks, a dtype cast on the device, and a
    whole HF checkpoint loaded onto the GPU equal to the same checkpoint loaded on the host."""
    from mod_b200.io.hf_loader import load_hf
    from mod_b200.io.safetensors import save_file
    from mod_b200.io.upload import StagedUploader
    from tests.test_io import _hf_from_fused

    up = StagedUploader(cuda, chunk_bytes=4096)
    src = torch.randn(257, 33)                              # 33,924 bytes: 9 chunks over both buffers
    got = up.upload(src[:, 1:])                             # non-contiguous source
    assert torch.equal(got.cpu(), src[:, 1:]) and up.nchunks == 9
    assert torch.equal(up.upload(src, torch.bfloat16).cpu(), src.bfloat16())
    cfg = get_preset("tiny-moe")
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=2)
    save_file(str(tmp_path / "model.safetensors"), _hf_from_fused(cfg, w), {})
    host = load_hf(cfg, str(tmp_path), device="cpu", dtype=torch.bfloat16)
    dev = load_hf(cfg, str(tmp_path), device=cuda, dtype=torch.bfloat16)
    for (n, a), (_, b) in zip(host.tensors(), dev.tensors()):
        assert b.is_cuda and torch.equal(a, b.cpu()), n
