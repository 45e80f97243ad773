"""Engine-backed model plugin: the reference's plugin lifecycle on top of LLMEngine.

Lifecycle (``pio/models/qwen3_0_6b/plugin.py:20-178``): ``__init__`` builds
metadata; ``initialize(**kwargs)`` applies config overrides, loads the
tokenizer and the model; ``infer`` / ``generate_text`` / ``infer_batch`` run
generation; ``get_model_info`` / ``get_model_parameters`` / ``cleanup``.
Differences: weights come from an HF checkpoint when ``model_path`` holds one
(random N(0, 0.02) otherwise, never a network download), and ``infer_batch``
uses the continuous batcher instead of a serial loop.
"""
from __future__ import annotations

import dataclasses
import logging
import os
from datetime import datetime
from typing import Any, Dict, List, Optional

import torch

from ..config.models import ModelConfig
from ..config.presets import get_preset
from ..engine.sequence import SamplingParams
from .interfaces import PluginMetadata, PluginType, TextModelPluginInterface

log = logging.getLogger("mod_b200.plugin")

_RUNTIME_KEYS = {"device", "backend", "max_batch", "max_model_len", "max_prefill_tokens", "seed", "model_path",
                 "use_graphs", "kv_mem_fraction", "max_new_tokens", "dtype", "prefix_caching",
                 "prefill_chunk", "offload", "offload_layers", "tp", "quantization"}


class EnginePlugin(TextModelPluginInterface):
    preset: str = "tiny-dense"
    display_name: str = "model"
    family: str = "Qwen"
    architecture: str = "Qwen3 Transformer"
    size: str = ""
    modalities = ("text",)
    # model-specific behaviour, set by each plugin
    thinking_default: bool = False       # chat replies open with a <think> block unless the caller says otherwise
    gpu_runtime_defaults: Dict[str, Any] = {}  # applied when the model runs on the sm_100a backend
    fim_tokens: Optional[tuple] = None   # (prefix, suffix, middle) markers of a fill-in-the-middle code model

    def __init__(self):
        cfg = get_preset(self.preset)
        self._config: ModelConfig = cfg if isinstance(cfg, ModelConfig) else cfg.text
        self._full_config = cfg
        md = PluginMetadata(name=self.display_name, version="1.0.0", author="mod_b200",
                            description=f"{self.display_name} on the mod_b200 B200 engine",
                            plugin_type=PluginType.MODEL_COMPONENT, dependencies=["torch"],
                            compatibility={"python_version": ">=3.10", "compute_capability": "10.0"},
                            model_architecture=self.architecture, model_size=self.size,
                            supported_modalities=list(self.modalities), license="Apache-2.0",
                            tags=[self.family.lower(), self.size.lower()], model_family=self.family,
                            num_parameters=self._config.num_params(), created_at=datetime.now(),
                            updated_at=datetime.now())
        super().__init__(md)
        self.runtime: Dict[str, Any] = {"device": "cuda" if torch.cuda.is_available() else "cpu",
                                        "backend": "native" if torch.cuda.is_available() else "torch",
                                        "max_batch": 8, "max_model_len": 2048, "seed": 0, "max_new_tokens": 10}
        self.engine = None
        self.tokenizer = None
        self.batch_manager = None

    # ------------------------------------------------------------------ lifecycle
    def initialize(self, **kwargs) -> bool:
        try:
            fields = {f.name for f in dataclasses.fields(ModelConfig)}
            for k, v in kwargs.items():
                if k.startswith("vision_") and hasattr(getattr(self._full_config, "vision", None), k[7:]):
                    setattr(self._full_config.vision, k[7:], v)
                elif k in _RUNTIME_KEYS or k == "image_size":
                    self.runtime[k] = v
                elif k in fields:
                    setattr(self._config, k, v)
                elif self._full_config is not self._config and hasattr(self._full_config, k):
                    setattr(self._full_config, k, v)
                else:
                    log.warning("%s: ignoring unknown option %s", self.display_name, k)
            if self.runtime["device"] == "cpu" and self.runtime["backend"] == "native":
                self.runtime["backend"] = "torch"
            if self.runtime["backend"] == "native":
                for k, v in self.gpu_runtime_defaults.items():
                    if k == "quantization" and int(self.runtime.get("tp", 1)) > 1:
                        continue  # tensor parallelism runs bf16 weights
                    if k not in kwargs:
                        self.runtime[k] = v
            from ..io.tokenizer import load_tokenizer

            self.tokenizer = load_tokenizer(self.runtime.get("model_path"))
            self.load_model()
            from .managers import BatchManager

            self.batch_manager = BatchManager(self)
            self._initialized = True
            return True
        except Exception as e:  # the reference reports False rather than raising
            log.error("%s: initialization failed: %s", self.display_name, e)
            return False

    def load_model(self, config: Optional[ModelConfig] = None):
        from ..engine.llm_engine import LLMEngine

        if config is not None:
            self._config = config
        rt = self.runtime
        dev = torch.device(rt["device"])
        dtype = torch.float32 if rt["backend"] in ("cpu",) or dev.type == "cpu" else torch.bfloat16
        weights = None
        path = rt.get("model_path")
        if not (path and os.path.isdir(path) and any(f.endswith(".safetensors") for f in os.listdir(path))):
            path = None  # random-init weights from the runtime seed
            from ..models.weights import random_weights

            if int(rt.get("tp", 1)) <= 1:
                weights = random_weights(self._config, device=dev, dtype=dtype, seed=rt["seed"])
        # with a checkpoint the engine reads it itself, so a TP or EP rank maps only its own slices
        self.engine = LLMEngine(self._config, weights=weights, backend=rt["backend"], device=dev,
                                model_path=path, seed=rt["seed"],
                                tensor_parallel=int(rt.get("tp", 1)) > 1,
                                quantization=rt.get("quantization"),
                                max_batch=rt["max_batch"], max_model_len=rt["max_model_len"],
                                use_graphs=rt.get("use_graphs"),
                                prefix_caching=bool(rt.get("prefix_caching", False)),
                                prefill_chunk=int(rt.get("prefill_chunk", 0)) or None,
                                offload_layers=(int(rt.get("offload_layers", 0)) or
                                                ("auto" if rt.get("offload") else None)))
        return self.engine

    def cleanup(self) -> bool:
        self.engine = None
        self.batch_manager = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        return super().cleanup()

    # ------------------------------------------------------------------ inference
    def tokenize(self, text: str, **kwargs) -> List[int]:
        return self.tokenizer.encode(text)

    def detokenize(self, token_ids: List[int], **kwargs) -> str:
        return self.tokenizer.decode([int(t) for t in token_ids])

    def _params(self, max_new_tokens=None, **kw) -> SamplingParams:
        return SamplingParams(max_new_tokens=max_new_tokens or self.runtime["max_new_tokens"],
                              temperature=kw.get("temperature", 0.0), top_p=kw.get("top_p", 1.0),
                              top_k=kw.get("top_k", 0), eos_token_id=getattr(self.tokenizer, "eos_token_id", None),
                              ignore_eos=kw.get("ignore_eos", False))

    def generate_ids(self, prompts: List[List[int]], max_new_tokens: Optional[int] = None, **kw) -> List[List[int]]:
        if self.engine is None:
            self.load_model()
        return self.engine.generate([[int(t) for t in p] for p in prompts], self._params(max_new_tokens, **kw))

    def generate_text(self, prompt: str, max_new_tokens: int = 512, **kwargs) -> str:
        ids = self.tokenize(prompt) or [0]
        out = self.generate_ids([ids], max_new_tokens, **kwargs)[0]
        return self.detokenize(out)

    # ------------------------------------------------------------------ chat / code
    def format_chat(self, messages: List[Dict[str, str]], enable_thinking: Optional[bool] = None) -> str:
        """The model's chat prompt for ``messages`` (ChatML for the Qwen3 family)."""
        from ..io.prompts import apply_chat_template

        think = self.thinking_default if enable_thinking is None else enable_thinking
        return apply_chat_template(self.tokenizer, messages, enable_thinking=think)

    def chat(self, messages: List[Dict[str, str]], max_new_tokens: Optional[int] = None,
             enable_thinking: Optional[bool] = None, **kw) -> str:
        """One assistant reply to ``messages``; any think block is stripped from it."""
        from ..io.prompts import strip_thinking

        text = self.format_chat(messages, enable_thinking)
        return strip_thinking(self.generate_text(text, max_new_tokens or self.runtime["max_new_tokens"], **kw)).strip()

    def format_fim(self, prefix: str, suffix: str = "") -> str:
        """Fill-in-the-middle prompt: the code before and after the gap, then the
        marker after which the model writes the missing middle."""
        if self.fim_tokens is None:
            raise NotImplementedError(f"{self.display_name} is not a fill-in-the-middle code model")
        p, s, m = self.fim_tokens
        return f"{p}{prefix}{s}{suffix}{m}"

    def complete_code(self, prefix: str, suffix: str = "", max_new_tokens: Optional[int] = None, **kw) -> str:
        """The code that fills the gap between ``prefix`` and ``suffix``."""
        return self.generate_text(self.format_fim(prefix, suffix), max_new_tokens or self.runtime["max_new_tokens"], **kw)

    def infer(self, data: Any) -> Any:
        """str -> generated text; token ids [B, L] (tensor or lists) -> [B, L + max_new_tokens]."""
        if isinstance(data, str):
            return self.generate_text(data, self.runtime["max_new_tokens"])
        if isinstance(data, torch.Tensor):
            rows = data.long().tolist() if data.dim() == 2 else [data.long().tolist()]
            outs = self.generate_ids(rows, ignore_eos=True)
            return torch.tensor([r + o for r, o in zip(rows, outs)], dtype=torch.long)
        if isinstance(data, (list, tuple)) and data and isinstance(data[0], (list, tuple)):
            outs = self.generate_ids(list(data), ignore_eos=True)
            return [list(r) + o for r, o in zip(data, outs)]
        raise TypeError(f"unsupported input {type(data)}")

    def infer_batch(self, requests: List[Any]) -> List[Any]:
        prompts = [self.tokenize(r) if isinstance(r, str) else list(r) for r in requests]
        outs = self.generate_ids(prompts, self.runtime["max_new_tokens"])
        return [self.detokenize(o) if isinstance(r, str) else o for r, o in zip(requests, outs)]

    # ------------------------------------------------------------------ info
    def get_model_info(self) -> Dict[str, Any]:
        c = self._config
        return {"name": self.display_name, "architecture": self.architecture, "parameters": c.num_params(),
                "active_parameters": c.active_params(), "hidden_size": c.hidden_size,
                "num_attention_heads": c.num_attention_heads, "num_key_value_heads": c.num_key_value_heads,
                "num_hidden_layers": c.num_hidden_layers, "num_experts": c.num_experts,
                "backend": self.runtime["backend"], "device": str(self.runtime["device"])}

    def get_model_parameters(self) -> Dict[str, Any]:
        return {"total_parameters": self._config.num_params(), "active_parameters": self._config.active_params()}

    def get_model_config_template(self) -> ModelConfig:
        cfg = get_preset(self.preset)
        return cfg if isinstance(cfg, ModelConfig) else cfg.text

    def validate_model_compatibility(self, config: Any) -> bool:
        return isinstance(config, ModelConfig) and config.model_type == self._config.model_type
