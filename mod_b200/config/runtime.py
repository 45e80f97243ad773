"""Runtime configuration, generation configuration, config-file loading.

Load order: defaults -> file (JSON or YAML) -> environment (``MB_*``; the
``PIO_*`` names of the same fields are read too, ``MB_*`` winning) -> explicit
overrides (CLI), then validation.  Named profiles mirror the reference's
presets (``pio/common/config/unified_config_manager.py:484-534``: performance,
memory_efficient, balanced).  The reference's loader/merge/validator live in
``pio/common/config/config_loader.py:17-154`` and
``pio/common/config/config_validator.py:20-154``.
"""
from __future__ import annotations

import copy
import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


@dataclass
class GenerationConfig:
    """Sampling defaults (``pio/common/config/generation_config.py:5-54``)."""

    max_new_tokens: int = 512
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0
    eos_token_id: Optional[int] = None
    do_sample: bool = False


@dataclass
class RuntimeConfig:
    """Where and how a model runs."""

    device: str = "cuda"
    backend: str = "native"              # native | torch | cpu
    dtype: str = "bfloat16"
    tp: int = 1                          # tensor parallel
    ep: int = 1                          # expert parallel
    pp: int = 1                          # pipeline stages
    dp: int = 1                          # data-parallel replicas
    kv_block_size: int = 16
    max_batch: int = 128
    max_model_len: int = 4096
    max_prefill_tokens: int = 16384
    kv_mem_fraction: float = 0.85
    cuda_graphs: bool = True
    comm: str = "fused"                  # fused (in-kernel NVLink) | nccl
    comm_timeout_s: float = 2.0          # bounded device waits
    debug_bounds: bool = False
    seed: int = 0
    threads: int = 0                     # CPU backend OpenMP threads (0: default)
    offload: bool = False                # hybrid CPU/GPU weight streaming (layer count from the planner)
    offload_layers: int = 0              # >0: stream this many trailing layers from pinned host memory
    prefix_caching: bool = False         # share KV blocks of common prompt prefixes
    prefill_chunk: int = 0               # >0: prefill prompts in chunks of this many tokens
    extra: Dict[str, Any] = field(default_factory=dict)


PROFILES: Dict[str, Dict[str, Any]] = {
    "performance": {"cuda_graphs": True, "kv_mem_fraction": 0.9, "comm": "fused"},
    "memory_efficient": {"kv_mem_fraction": 0.5, "max_batch": 32, "offload": True},
    "balanced": {"kv_mem_fraction": 0.8, "max_batch": 64},
}

_VALID = {
    "backend": {"native", "torch", "cpu"},
    "comm": {"fused", "nccl"},
    "dtype": {"bfloat16", "float16", "float32"},
}


class ConfigError(ValueError):
    pass


def validate(cfg: RuntimeConfig) -> RuntimeConfig:
    errs: List[str] = []
    for k, allowed in _VALID.items():
        if getattr(cfg, k) not in allowed:
            errs.append(f"{k}={getattr(cfg, k)!r} not in {sorted(allowed)}")
    for k in ("tp", "ep", "pp", "dp", "max_batch", "max_model_len", "kv_block_size", "max_prefill_tokens"):
        if getattr(cfg, k) < 1:
            errs.append(f"{k} must be >= 1")
    if not 0.0 < cfg.kv_mem_fraction <= 1.0:
        errs.append("kv_mem_fraction must be in (0, 1]")
    if cfg.kv_block_size != 16 and cfg.backend == "native":
        errs.append("the native kernels use kv_block_size 16")
    if cfg.backend == "cpu" and cfg.device != "cpu":
        errs.append("backend 'cpu' needs device 'cpu'")
    if errs:
        raise ConfigError("; ".join(errs))
    return cfg


def deep_merge(base: Dict[str, Any], over: Dict[str, Any]) -> Dict[str, Any]:
    out = copy.deepcopy(base)
    for k, v in over.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = deep_merge(out[k], v)
        else:
            out[k] = copy.deepcopy(v)
    return out


def load_file(path: str) -> Dict[str, Any]:
    with open(path) as f:
        text = f.read()
    if path.endswith((".yaml", ".yml")):
        import yaml

        return yaml.safe_load(text) or {}
    return json.loads(text)


def _coerce(value: str, typ):
    if typ is bool or typ == "bool":
        return value.lower() in ("1", "true", "yes", "on")
    if typ is int or typ == "int":
        return int(value)
    if typ is float or typ == "float":
        return float(value)
    return value


def from_env(prefix: str = "MB_") -> Dict[str, Any]:
    out = {}
    for f in dataclasses.fields(RuntimeConfig):
        key = prefix + f.name.upper()
        if key in os.environ and f.name != "extra":
            out[f.name] = _coerce(os.environ[key], f.type)
    return out


def load_runtime(path: Optional[str] = None, profile: Optional[str] = None,
                 overrides: Optional[Dict[str, Any]] = None, env: bool = True) -> RuntimeConfig:
    """defaults -> profile -> file -> env -> overrides, validated."""
    d = dataclasses.asdict(RuntimeConfig())
    if profile:
        if profile not in PROFILES:
            raise ConfigError(f"unknown profile {profile!r}; known: {sorted(PROFILES)}")
        d = deep_merge(d, PROFILES[profile])
    if path:
        data = load_file(path)
        d = deep_merge(d, data.get("runtime", data))
    if env:
        d = deep_merge(d, from_env("PIO_"))
        d = deep_merge(d, from_env())
    if overrides:
        d = deep_merge(d, {k: v for k, v in overrides.items() if v is not None})
    known = {f.name for f in dataclasses.fields(RuntimeConfig)}
    extra = {k: v for k, v in d.items() if k not in known}
    kw = {k: v for k, v in d.items() if k in known}
    kw.setdefault("extra", {}).update(extra)
    return validate(RuntimeConfig(**kw))


def save(cfg, path: str) -> None:
    d = dataclasses.asdict(cfg)
    with open(path, "w") as f:
        if path.endswith((".yaml", ".yml")):
            import yaml

            yaml.safe_dump(d, f)
        else:
            json.dump(d, f, indent=2)
