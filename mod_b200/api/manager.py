"""Plugin manager, secondary-plugin registry and model factory.

* :class:`PluginManager` discovers model plugins from ``plugin_manifest.json``
  files (``entry_point = "module:factory"``), registers, activates
  (initialize with options), executes plugin methods and tracks the hardware
  backends.  Counterpart of ``pio/plugins/manager.py:24-235``, which executes
  every ``plugin.py`` it finds and crashes on a missing
  ``HardwareAnalyzer.get_hardware_info``.
* :class:`SecondaryPluginManager` - typed registry of extension plugins
  (memory manager, distributed execution, kernel fusion, ...), as
  ``pio/plugins/secondary_manager.py:14-165``.
* :class:`ModelFactory` - name normalisation -> plugin
  (``pio/core/model_factory.py:26-246``).
"""
from __future__ import annotations

import enum
import glob
import importlib
import json
import logging
import os
import re
from typing import Any, Callable, Dict, List, Optional

from .backends import available_backends, create_backend, probe_system
from .interfaces import ModelPluginInterface, PluginMetadata

log = logging.getLogger("mod_b200.plugins")
PLUGIN_ROOT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "models", "plugins")


def _normalise(name: str) -> str:
    return re.sub(r"[^a-z0-9]", "", name.lower())


class PluginManager:
    def __init__(self, plugin_dirs: Optional[List[str]] = None):
        self.plugin_dirs = plugin_dirs or [PLUGIN_ROOT]
        self.manifests: Dict[str, Dict[str, Any]] = {}
        self.factories: Dict[str, Callable[[], ModelPluginInterface]] = {}
        self.plugins: Dict[str, ModelPluginInterface] = {}
        self.active: Dict[str, ModelPluginInterface] = {}
        self.backends: Dict[str, Any] = {}

    # ------------------------------------------------------------------ discovery
    def discover_and_load_plugins(self) -> List[str]:
        found = []
        for d in self.plugin_dirs:
            for mf in sorted(glob.glob(os.path.join(d, "*", "plugin_manifest.json"))):
                try:
                    with open(mf) as f:
                        m = json.load(f)
                    self.register_manifest(m)
                    found.append(m["name"])
                except Exception as e:
                    log.warning("skipping plugin manifest %s: %s", mf, e)
        return found

    def register_manifest(self, manifest: Dict[str, Any]) -> None:
        PluginMetadata.from_manifest(manifest)  # validates the fields
        name = manifest["name"]
        self.manifests[name] = manifest

        def factory(ep=manifest["entry_point"]):
            mod, _, fn = ep.partition(":")
            return getattr(importlib.import_module(mod), fn)()

        self.factories[name] = factory

    def register_plugin(self, plugin: ModelPluginInterface) -> None:
        self.plugins[plugin.metadata.name] = plugin

    def resolve(self, name: str) -> str:
        key = _normalise(name)
        for n, m in self.manifests.items():
            aliases = {_normalise(n), _normalise(m.get("preset", "")), _normalise(os.path.basename(m.get("entry_point", "").split(":")[0].rsplit(".", 1)[0]))}
            if key in aliases:
                return n
        for n in self.plugins:
            if _normalise(n) == key:
                return n
        raise KeyError(f"no plugin named {name!r}; available: {sorted(self.manifests) + sorted(self.plugins)}")

    def list_plugins(self) -> List[Dict[str, Any]]:
        out = [dict(m, active=n in self.active) for n, m in self.manifests.items()]
        out += [dict(p.metadata.to_dict(), active=n in self.active) for n, p in self.plugins.items()
                if n not in self.manifests]
        return out

    # ------------------------------------------------------------------ lifecycle
    def get_plugin(self, name: str) -> ModelPluginInterface:
        n = self.resolve(name)
        if n not in self.plugins:
            self.plugins[n] = self.factories[n]()
        return self.plugins[n]

    def activate_plugin(self, name: str, **options) -> bool:
        p = self.get_plugin(name)
        ok = p.initialize(**options)
        if ok:
            self.active[p.metadata.name] = p
        return ok

    def deactivate_plugin(self, name: str) -> None:
        n = self.resolve(name)
        p = self.active.pop(n, None)
        if p is not None:
            p.cleanup()

    def execute_plugin(self, name: str, method: str = "infer", *args, **kwargs):
        n = self.resolve(name)
        if n not in self.active:
            raise RuntimeError(f"plugin {n} is not active")
        return getattr(self.active[n], method)(*args, **kwargs)

    # ------------------------------------------------------------------ backends
    def load_hardware_backends(self) -> Dict[str, Any]:
        for spec in available_backends():
            try:
                b = create_backend(spec)
                if b.initialize():
                    self.backends[spec] = b
            except Exception as e:  # a backend that cannot start is reported, not fatal
                log.warning("backend %s unavailable: %s", spec, e)
        return self.backends

    def system_info(self) -> Dict[str, Any]:
        return probe_system()


_MANAGER: Optional[PluginManager] = None


def get_plugin_manager() -> PluginManager:
    global _MANAGER
    if _MANAGER is None:
        _MANAGER = PluginManager()
        _MANAGER.discover_and_load_plugins()
    return _MANAGER


class SecondaryPluginType(enum.Enum):
    MEMORY_MANAGER = "memory_manager"
    DISTRIBUTED_EXECUTION = "distributed_execution"
    COMPRESSION = "compression"
    SECURITY = "security"
    KERNEL_FUSION = "kernel_fusion"
    ADAPTIVE_BATCHING = "adaptive_batching"
    MODEL_SURGERY = "model_surgery"
    PIPELINE = "pipeline"
    SHARDING = "sharding"


class SecondaryPlugin:
    """A secondary (feature) plugin: a named factory whose ``initialize(**kw)``
    builds the component, ``execute(*a, **kw)`` calls it, ``cleanup()`` drops it.
    Same lifecycle as the reference's ``SecondaryPluginInterface``
    (``pio/plugins/secondary_manager.py:20-66``)."""

    def __init__(self, name: str, factory: Callable[..., Any], description: str = "",
                 call: Optional[Callable[..., Any]] = None):
        self.name, self.factory, self.description = name, factory, description
        self._call = call
        self.instance: Any = None

    def initialize(self, **kw) -> bool:
        try:
            self.instance = self.factory(**kw)
        except Exception as e:  # reported as a failed activation, like the reference
            logging.getLogger("mod_b200.plugins").error("secondary plugin %s: %s", self.name, e)
            self.instance = None
            return False
        return True

    def execute(self, *a, **kw) -> Any:
        if self._call is not None:
            return self._call(self.instance, *a, **kw)
        return self.instance(*a, **kw) if callable(self.instance) else self.instance

    def cleanup(self) -> bool:
        self.instance = None
        return True


class SecondaryPluginManager:
    """Registry of secondary plugins by kind and name, with activation.

    The default registrations (``register_defaults``) are the components this
    engine actually uses: the unified memory manager, the two communication
    backends (fused NVLink kernels / NCCL), adaptive admission, the pipeline
    stage executor, the placement planner, the sm_100a kernel backend, int8
    weight-only compression, memory budgets and layer streaming (the hybrid
    CPU/GPU scheduler).  The reference's manager keeps one plugin per kind and
    registers none (``pio/plugins/secondary_manager.py:69-165``)."""

    def __init__(self, defaults: bool = False):
        self._reg: Dict[SecondaryPluginType, Dict[str, Any]] = {t: {} for t in SecondaryPluginType}
        self.active: Dict[SecondaryPluginType, str] = {}
        if defaults:
            register_defaults(self)

    def register(self, kind: SecondaryPluginType, name: str, obj: Any) -> None:
        self._reg[kind][name] = obj

    def get(self, kind: SecondaryPluginType, name: str) -> Any:
        return self._reg[kind][name]

    def list(self, kind: Optional[SecondaryPluginType] = None) -> Dict[str, List[str]]:
        kinds = [kind] if kind else list(SecondaryPluginType)
        return {k.value: sorted(self._reg[k]) for k in kinds}

    # reference-style lifecycle: one active plugin per kind
    def register_plugin(self, kind: SecondaryPluginType, plugin: SecondaryPlugin) -> None:
        self.register(kind, plugin.name, plugin)

    def get_plugin(self, kind: SecondaryPluginType, name: Optional[str] = None) -> Optional[SecondaryPlugin]:
        name = name or self.active.get(kind)
        if name is None and len(self._reg[kind]) == 1:
            name = next(iter(self._reg[kind]))
        return self._reg[kind].get(name) if name else None

    def activate_plugin(self, kind: SecondaryPluginType, name: Optional[str] = None, **kw) -> bool:
        p = self.get_plugin(kind, name)
        if p is None or not p.initialize(**kw):
            return False
        self.active[kind] = p.name
        return True

    def deactivate_plugin(self, kind: SecondaryPluginType) -> bool:
        name = self.active.pop(kind, None)
        if name is None:
            return False
        return self._reg[kind][name].cleanup()

    def execute_plugin(self, kind: SecondaryPluginType, *a, **kw) -> Any:
        name = self.active.get(kind)
        if name is None:
            return None
        return self._reg[kind][name].execute(*a, **kw)


def register_defaults(m: SecondaryPluginManager) -> SecondaryPluginManager:
    """Registers the engine's components as secondary plugins (imports are lazy)."""
    T = SecondaryPluginType

    def mem(device="cuda", **kw):
        from ..runtime.memory import UnifiedMemoryManager

        return UnifiedMemoryManager(device, **kw)

    def fused_comm(parallelism="ep", **kw):
        from ..parallel import ep, tp

        return ep.FusedEPMoE if parallelism == "ep" else tp.FusedTP

    def nccl_comm(parallelism="ep", **kw):
        from ..parallel import ep, tp

        return ep.NcclEPMoE if parallelism == "ep" else tp.NcclTP

    def nvls_comm(parallelism="ep", **kw):
        from ..parallel import ep_agrs, tp

        return ep_agrs.AgRsEPMoE if parallelism == "ep" else tp.NvlsTP

    def admission(**kw):
        from .managers import AdaptiveAdmission

        return AdaptiveAdmission(**kw)

    def pipeline(**kw):
        from ..parallel.pipeline import PipelineExecutor

        return PipelineExecutor

    def planner(**kw):
        from ..parallel.planner import plan

        return plan

    def kernels(**kw):
        from ..models.backend import make_backend

        return make_backend("native")

    def int8(**kw):
        from ..ops.quant import quantize_model

        return quantize_model

    def budgets(device="cuda", **kw):
        from ..runtime.memory import UnifiedMemoryManager

        return UnifiedMemoryManager(device, **kw)

    def streaming(**kw):
        from ..runtime.offload import enable_streaming

        return enable_streaming

    m.register_plugin(T.MEMORY_MANAGER, SecondaryPlugin(
        "unified", mem, "one owner of device memory per rank: KV pool sizing, region budgets, KV swap",
        call=lambda inst, *a, **k: inst.report()))
    m.register_plugin(T.DISTRIBUTED_EXECUTION, SecondaryPlugin(
        "fused-nvlink", fused_comm, "in-kernel NVLink dispatch/combine (EP) and fused TP boundaries",
        call=lambda inst, *a, **k: inst(*a, **k) if a or k else inst))
    m.register_plugin(T.DISTRIBUTED_EXECUTION, SecondaryPlugin(
        "nvls", nvls_comm, "NVLink multicast: in-switch reduce + multicast stores (TP boundaries, EP decode)",
        call=lambda inst, *a, **k: inst(*a, **k) if a or k else inst))
    m.register_plugin(T.DISTRIBUTED_EXECUTION, SecondaryPlugin(
        "nccl", nccl_comm, "NCCL all-to-all / all-reduce with library GEMMs (baseline)",
        call=lambda inst, *a, **k: inst(*a, **k) if a or k else inst))
    m.register_plugin(T.ADAPTIVE_BATCHING, SecondaryPlugin(
        "adaptive-admission", admission, "admission control by measured step latency"))
    m.register_plugin(T.PIPELINE, SecondaryPlugin("stage-executor", pipeline, "micro-batched pipeline stages"))
    m.register_plugin(T.SHARDING, SecondaryPlugin("planner", planner, "TP/EP/PP/DP degrees and per-GPU bytes"))
    m.register_plugin(T.KERNEL_FUSION, SecondaryPlugin("sm100-native", kernels, "hand-written sm_100a kernels"))
    m.register_plugin(T.COMPRESSION, SecondaryPlugin("int8-weight-only", int8, "per-channel int8 projections"))
    m.register_plugin(T.SECURITY, SecondaryPlugin(
        "memory-budgets", budgets, "per-region byte budgets (OutOfBudget on overrun)",
        call=lambda inst, region, nbytes: inst.charge(region, nbytes)))
    m.register_plugin(T.MODEL_SURGERY, SecondaryPlugin(
        "layer-streaming", streaming, "stream trailing layers from pinned host memory (hybrid CPU/GPU)"))
    return m


_SECONDARY: Optional[SecondaryPluginManager] = None


def get_secondary_plugin_manager() -> SecondaryPluginManager:
    global _SECONDARY
    if _SECONDARY is None:
        _SECONDARY = SecondaryPluginManager(defaults=True)
    return _SECONDARY


class ModelFactory:
    """``create_model("qwen3-0.6b", **options)`` -> an initialised plugin."""

    def __init__(self, manager: Optional[PluginManager] = None):
        self.pm = manager or get_plugin_manager()

    def available(self) -> List[str]:
        return sorted(self.pm.manifests)

    def create_model(self, name: str, **options) -> ModelPluginInterface:
        p = self.pm.get_plugin(name)
        if not p.initialize(**options):
            raise RuntimeError(f"could not initialise {name}")
        self.pm.active[p.metadata.name] = p
        return p

    def register_model(self, name: str, factory: Callable[[], ModelPluginInterface], **manifest) -> None:
        p = factory()
        self.pm.plugins[name] = p


def create_model(name: str, **options) -> ModelPluginInterface:
    return ModelFactory().create_model(name, **options)
