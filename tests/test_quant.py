"""int8 weight-only quantisation (host side) and the torch-backend int8 engine path."""
import torch

from mod_b200.config import get_preset
from mod_b200.engine import SamplingParams
from mod_b200.engine.llm_engine import LLMEngine
from mod_b200.models.weights import random_weights
from mod_b200.ops.quant import Int8Weight, quantize_int8, quantize_model


def test_quantize_roundtrip_bound():
    torch.manual_seed(0)
    w = torch.randn(64, 96) * 0.03
    q = quantize_int8(w)
    assert q.q.dtype == torch.int8 and q.scale.shape == (64,)
    assert int(q.q.abs().max()) <= 127
    err = (q.dequant(torch.float32) - w).abs()
    # per-row error is at most half a quantisation step
    assert bool((err <= q.scale[:, None] * 0.5 + 1e-7).all())


def test_quantize_model_replaces_projections():
    cfg = get_preset("tiny-next")
    w = quantize_model(random_weights(cfg, device="cpu", dtype=torch.float32, seed=0))
    kinds = set()
    for L in w.layers:
        if L.attn is not None:
            assert isinstance(L.attn.qkv, Int8Weight) and isinstance(L.attn.o, Int8Weight)
            kinds.add("attn")
        if L.delta is not None:
            assert isinstance(L.delta.in_qkvz, Int8Weight) and isinstance(L.delta.out, Int8Weight)
            kinds.add("delta")
        if L.moe is not None:
            assert isinstance(L.moe.w13, Int8Weight) and isinstance(L.moe.w2, Int8Weight)
            assert not isinstance(L.moe.router, Int8Weight)
            kinds.add("moe")
    assert kinds == {"attn", "delta", "moe"}


def test_int8_engine_torch_backend_runs_close_to_bf16():
    cfg = get_preset("tiny-dense")
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
    logits = {}
    for quant in (None, "int8"):
        w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=4)
        eng = LLMEngine(cfg, weights=w, backend="torch", device="cpu", max_batch=2, max_model_len=64,
                        quantization=quant)
        rid = eng.add_request(prompt, SamplingParams(max_new_tokens=3, ignore_eos=True))
        while eng.has_unfinished():
            eng.step()
        assert len(eng.seqs[rid].output) == 3
        logits[quant] = eng.seqs[rid].output
    assert eng.quantization == "int8"
