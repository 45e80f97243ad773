"""safetensors reader/writer, HF-layout loader, tokenizer, prompt utilities."""
import json
import os

import pytest
import torch

from mod_b200.config import get_preset
from mod_b200.models.weights import random_weights

C = pytest.importorskip("mod_b200._cpu")
from mod_b200.io.safetensors import save_file  # noqa: E402


def test_safetensors_roundtrip_and_slices(tmp_path):
    p = str(tmp_path / "a.safetensors")
    t = {"a": torch.randn(8, 6), "b": torch.arange(10, dtype=torch.int64), "c": torch.randn(4, 4).bfloat16(),
         "d": torch.tensor([1, -2, 3], dtype=torch.int8)}
    save_file(p, t, {"k": "v"})
    f = C.SafeTensorsFile(p)
    assert sorted(f.keys()) == ["a", "b", "c", "d"] and f.metadata() == {"k": "v"}
    for k, v in t.items():
        assert torch.equal(f.get(k), v) and f.dtype(k) in ("F32", "I64", "BF16", "I8")
    assert torch.equal(f.get_slice("a", 0, 1, 2), t["a"][4:])
    assert torch.equal(f.get_slice("a", 1, 2, 3), t["a"][:, 4:])
    with pytest.raises(Exception):
        f.get_slice("a", 1, 0, 4)      # 6 not divisible by 4
    h = C.read_header(p)
    assert h["a"]["shape"] == [8, 6]


@pytest.mark.parametrize("corrupt", ["short", "hdrlen", "json", "offsets"])
def test_safetensors_rejects_corrupt_files(tmp_path, corrupt):
    p = str(tmp_path / "x.safetensors")
    save_file(p, {"a": torch.randn(4)}, {})
    raw = bytearray(open(p, "rb").read())
    if corrupt == "short":
        raw = raw[:5]
    elif corrupt == "hdrlen":
        raw[0:8] = (10**12).to_bytes(8, "little")
    elif corrupt == "json":
        raw[8] = ord("[")
    else:
        n = int.from_bytes(raw[:8], "little")
        hdr = json.loads(raw[8:8 + n])
        hdr["a"]["data_offsets"] = [0, 10**9]
        s = json.dumps(hdr).encode()
        s += b" " * (n - len(s))
        raw[8:8 + n] = s[:n]
    open(p, "wb").write(bytes(raw))
    with pytest.raises(Exception):
        C.SafeTensorsFile(p)


def _hf_from_fused(cfg, w):
    """Writes fused random weights back out in the HF naming (dense Qwen3 / MoE)."""
    H, D, Hq, Hkv = cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    out = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm}
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = w.lm_head
    for i, L in enumerate(w.layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = L.in_norm
        out[p + "post_attention_layernorm.weight"] = L.post_norm
        q, k, v = L.attn.qkv.split([Hq * D, Hkv * D, Hkv * D])
        out.update({p + "self_attn.q_proj.weight": q, p + "self_attn.k_proj.weight": k,
                    p + "self_attn.v_proj.weight": v, p + "self_attn.o_proj.weight": L.attn.o,
                    p + "self_attn.q_norm.weight": L.attn.q_norm, p + "self_attn.k_norm.weight": L.attn.k_norm})
        if L.moe is not None:
            I = cfg.moe_intermediate_size
            out[p + "mlp.gate.weight"] = L.moe.router
            for e in range(cfg.num_experts):
                g, u = L.moe.w13[e * 2 * I:(e + 1) * 2 * I].split([I, I])
                out[p + f"mlp.experts.{e}.gate_proj.weight"] = g
                out[p + f"mlp.experts.{e}.up_proj.weight"] = u
                out[p + f"mlp.experts.{e}.down_proj.weight"] = L.moe.w2[e * H:(e + 1) * H]
        else:
            I = cfg.intermediate_size
            g, u = L.mlp.gate_up.split([I, I])
            out.update({p + "mlp.gate_proj.weight": g, p + "mlp.up_proj.weight": u, p + "mlp.down_proj.weight": L.mlp.down})
    return {k: v.contiguous() for k, v in out.items()}


@pytest.mark.parametrize("name", ["tiny-dense", "tiny-moe"])
def test_hf_loader_roundtrip(tmp_path, name):
    from mod_b200.io.hf_loader import load_hf, load_weights, save_weights
    from mod_b200.models import oracle

    cfg = get_preset(name)
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=3)
    d = tmp_path / "ckpt"
    d.mkdir()
    save_file(str(d / "model.safetensors"), _hf_from_fused(cfg, w), {})
    w2 = load_hf(cfg, str(d), device="cpu", dtype=torch.float32)
    ids = torch.tensor([[1, 5, 9, 33]])
    torch.testing.assert_close(oracle.forward(cfg, w2, ids), oracle.forward(cfg, w, ids))
    # expert-parallel slice loads only its experts
    if cfg.is_moe:
        w3 = load_hf(cfg, str(d), device="cpu", dtype=torch.float32, expert_range=(4, 8))
        I = cfg.moe_intermediate_size
        assert torch.equal(w3.layers[0].moe.w13, w.layers[0].moe.w13[4 * 2 * I:8 * 2 * I])
    # our own fused format
    save_weights(w, str(tmp_path / "fused.safetensors"), cfg)
    w4 = load_weights(str(tmp_path / "fused.safetensors"), cfg, device="cpu")
    torch.testing.assert_close(oracle.forward(cfg, w4, ids), oracle.forward(cfg, w, ids))


def test_bpe_tokenizer_roundtrip(tmp_path):
    from mod_b200.io.tokenizer import ByteBPETokenizer, SimpleTokenizer, byte_to_unicode, load_tokenizer

    b2u = byte_to_unicode()
    vocab = {c: i for i, c in enumerate(b2u.values())}
    merges = [("h", "e"), ("l", "l"), ("he", "ll"), ("Ġ", "w")]
    for a, b in merges:
        vocab.setdefault(a + b, len(vocab))
    vocab["<|im_end|>"] = len(vocab)
    (tmp_path / "vocab.json").write_text(json.dumps(vocab))
    (tmp_path / "merges.txt").write_text("#version: 0.2\n" + "\n".join(f"{a} {b}" for a, b in merges))
    tok = load_tokenizer(str(tmp_path))
    assert isinstance(tok, ByteBPETokenizer)
    for text in ["hello world", "héllo 123 ✓\nnew line", ""]:
        assert tok.decode(tok.encode(text)) == text
    ids = tok.encode("hello")
    assert vocab["hell"] in ids
    s = SimpleTokenizer()
    assert s.decode(s.encode("abc é")) == "abc é"


def test_prompt_utils():
    from mod_b200.io import prompts

    assert prompts.format_math_prompt("1+1?").endswith(prompts.MATH_SUFFIX)
    assert prompts.format_math_prompt(prompts.format_math_prompt("q")).count("boxed") == 1
    h = prompts.format_history([{"role": "user", "content": "hi"},
                                {"role": "assistant", "content": "<think>hmm</think> Hello"}])
    assert h[1]["content"] == "Hello"
    t = prompts.apply_chat_template(None, [{"role": "user", "content": "x"}])
    assert t == "<|im_start|>user\nx<|im_end|>\n<|im_start|>assistant\n<think>\n"


def test_hf_loader_tensor_parallel_slices(tmp_path):
    """load_hf(tp=(r, N)) reads each rank's projection slices from the mapping and
    gives exactly shard_weights() of the full load, for every rank."""
    from mod_b200.io.hf_loader import load_hf
    from mod_b200.models.tp_decoder import shard_weights

    cfg = get_preset("tiny-dense")
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=5)
    d = tmp_path / "ckpt"
    d.mkdir()
    save_file(str(d / "model.safetensors"), _hf_from_fused(cfg, w), {})
    full = load_hf(cfg, str(d), device="cpu", dtype=torch.float32)
    world = 2
    for rank in range(world):
        got = load_hf(cfg, str(d), device="cpu", dtype=torch.float32, tp=(rank, world))
        want = shard_weights(cfg, full, rank, world)
        for a, b in zip(got.layers, want.layers):
            assert torch.equal(a.attn.qkv, b.attn.qkv)
            assert torch.equal(a.attn.o, b.attn.o)
            assert torch.equal(a.mlp.gate_up, b.mlp.gate_up)
            assert torch.equal(a.mlp.down, b.mlp.down)
            assert a.attn.o.is_contiguous() and a.mlp.down.is_contiguous()
        assert torch.equal(got.embed, want.embed) and torch.equal(got.lm_head, want.lm_head)
