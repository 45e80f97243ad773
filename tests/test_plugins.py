"""Plugin API: discovery from manifests, lifecycle, inference through the
engine, factory name resolution (reference contract: initialise with small
kwargs -> infer(Tensor [1, 2]) -> shape [1, 2 + 10] -> cleanup)."""
import pytest
import torch

from mod_b200.api import ModelFactory, PluginManager, PluginMetadata, SecondaryPluginManager, SecondaryPluginType

SMALL = dict(device="cpu", backend="torch", hidden_size=128, intermediate_size=256, num_hidden_layers=1,
             num_attention_heads=2, num_key_value_heads=1, head_dim=64, vocab_size=300, max_batch=2,
             max_model_len=64)
NAMES = ["Qwen3-0.6B", "Qwen3-4B-Instruct-2507", "Qwen3-Coder-30B", "Qwen3-Coder-Next", "GLM-4.7-Flash"]


def test_discovery_lists_all_models():
    pm = PluginManager()
    found = pm.discover_and_load_plugins()
    assert set(NAMES + ["Qwen3-VL-2B"]) <= set(found)
    for m in pm.list_plugins():
        md = PluginMetadata.from_manifest(m)
        assert md.name and md.model_architecture
    assert pm.resolve("qwen3_0_6b") == "Qwen3-0.6B"
    assert pm.resolve("qwen3-30b-a3b") == "Qwen3-Coder-30B"
    with pytest.raises(KeyError):
        pm.resolve("no-such-model")


@pytest.mark.parametrize("name", NAMES)
def test_plugin_lifecycle_small(name):
    pm = PluginManager()
    pm.discover_and_load_plugins()
    extra = {}
    if name in ("Qwen3-Coder-30B", "Qwen3-Coder-Next"):
        extra = dict(num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128)
    if name == "Qwen3-Coder-Next":
        extra.update(num_hidden_layers=2, layer_types=["linear_attention", "full_attention"], linear_num_key_heads=1,
                     linear_num_value_heads=2, linear_key_head_dim=32, linear_value_head_dim=32,
                     shared_expert_intermediate_size=128)
    assert pm.activate_plugin(name, **{**SMALL, **extra})
    p = pm.get_plugin(name)
    out = pm.execute_plugin(name, "infer", torch.tensor([[1, 2]]))
    assert tuple(out.shape) == (1, 12)
    assert isinstance(p.generate_text("hi", max_new_tokens=3), str)
    res = p.infer_batch(["a", "bc", "def"])
    assert len(res) == 3
    info = p.get_model_info()
    assert info["num_hidden_layers"] == SMALL["num_hidden_layers"] or name == "Qwen3-Coder-Next"
    pm.deactivate_plugin(name)
    assert not p.is_initialized


def test_vl_plugin_image_inference_matches_oracle():
    from mod_b200.models import vl

    pm = PluginManager()
    pm.discover_and_load_plugins()
    assert pm.activate_plugin("Qwen3-VL-2B", **SMALL, image_size=64, vision_hidden_size=64,
                              vision_num_hidden_layers=1, vision_num_attention_heads=2, vision_intermediate_size=128,
                              vision_out_hidden_size=128, image_token_id=299)
    p = pm.get_plugin("Qwen3-VL-2B")
    torch.manual_seed(0)
    img = torch.rand(3, 64, 64)
    out = p.infer(([5, 6, 7], img))
    assert len(out) == 4 + 3 + 10       # 64x64 image: 4x4 patches -> 4 merged visual tokens
    cfg = p._full_config
    ids = torch.tensor([p.vl.prompt_with_image([5, 6, 7])])
    ref = vl.oracle_forward(cfg, p.vl.w, p.vl.vw, img[None], ids, 64)
    assert out[ids.shape[1]] == int(ref[0, -1].argmax())


def test_secondary_registry_and_factory():
    s = SecondaryPluginManager()
    s.register(SecondaryPluginType.MEMORY_MANAGER, "unified", object())
    assert s.list(SecondaryPluginType.MEMORY_MANAGER) == {"memory_manager": ["unified"]}
    f = ModelFactory(PluginManager())
    f.pm.discover_and_load_plugins()
    m = f.create_model("qwen3-0.6b", **SMALL)
    assert m.is_initialized


def _plugin(name):
    pm = PluginManager()
    pm.discover_and_load_plugins()
    return pm, pm.get_plugin(name)


def test_plugin_specific_chat_layouts():
    """Thinking defaults differ per model (Qwen3-0.6B hybrid-thinking, 4B-Instruct-2507
    non-thinking); GLM has its own chat layout."""
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    _, small = _plugin("Qwen3-0.6B")
    assert small.format_chat(msgs).endswith("<|im_start|>assistant\n<think>\n")
    assert small.format_chat(msgs, enable_thinking=False).endswith("<|im_start|>assistant\n")
    _, inst = _plugin("Qwen3-4B-Instruct-2507")
    assert inst.format_chat(msgs).endswith("<|im_start|>assistant\n")
    _, glm = _plugin("GLM-4.7-Flash")
    assert glm.format_chat(msgs) == "[gMASK]<sop><|system|>\nbe brief<|user|>\nhi/nothink<|assistant|>\n"
    assert "/nothink" not in glm.format_chat(msgs, enable_thinking=True)


def test_coder_plugins_fill_in_the_middle_and_next_defaults():
    pm, coder = _plugin("Qwen3-Coder-30B")
    assert coder.format_fim("def f(x):\n    ", "\n    return y") == \
        "<|fim_prefix|>def f(x):\n    <|fim_suffix|>\n    return y<|fim_middle|>"
    _, small = _plugin("Qwen3-0.6B")
    with pytest.raises(NotImplementedError):
        small.format_fim("a")
    assert pm.activate_plugin("Qwen3-Coder-30B", **SMALL, num_experts=8, num_experts_per_tok=2,
                              moe_intermediate_size=128)
    assert isinstance(coder.complete_code("def f(", "):", max_new_tokens=3), str)
    assert isinstance(coder.chat([{"role": "user", "content": "x"}], max_new_tokens=3), str)
    pm.deactivate_plugin("Qwen3-Coder-30B")
    # Qwen3-Next on the sm_100a backend defaults to int8 projections and chunked prefill; an explicit
    # option wins, and the CPU-side torch backend keeps bf16/fp32 weights
    _, nxt = _plugin("Qwen3-Coder-Next")
    assert nxt.gpu_runtime_defaults == {"quantization": "int8", "prefill_chunk": 8192}
    assert "quantization" not in nxt.runtime
