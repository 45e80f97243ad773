"""Plugin interfaces.

Same public names and methods as the reference
(``pio/common/interfaces/improved_base_plugin_interface.py:5-62``):
``PluginType``, ``PluginMetadata``, ``ModelPluginInterface``,
``TextModelPluginInterface`` (``infer``, ``generate_text``, ``load_model``,
``tokenize``, ``detokenize``, ``infer_batch``), so code written against the
reference's plugin API keeps working.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from datetime import datetime
from enum import Enum
from typing import Any, Dict, List, Optional


class PluginType(Enum):
    MODEL_COMPONENT = "MODEL_COMPONENT"
    HARDWARE_BACKEND = "HARDWARE_BACKEND"
    SECONDARY = "SECONDARY"


@dataclass
class PluginMetadata:
    name: str
    version: str
    author: str
    description: str
    plugin_type: PluginType
    dependencies: List[str] = field(default_factory=list)
    compatibility: Dict[str, str] = field(default_factory=dict)
    model_architecture: str = ""
    model_size: str = ""
    required_memory_gb: float = 0.0
    supported_modalities: Optional[List[str]] = None
    license: str = ""
    tags: Optional[List[str]] = None
    model_family: str = ""
    num_parameters: int = 0
    test_coverage: float = 0.0
    validation_passed: bool = False
    created_at: Any = None
    updated_at: Any = None

    def to_dict(self) -> Dict[str, Any]:
        d = asdict(self)
        d["plugin_type"] = self.plugin_type.value
        for k in ("created_at", "updated_at"):
            if isinstance(d[k], datetime):
                d[k] = d[k].isoformat()
        return d

    @classmethod
    def from_manifest(cls, m: Dict[str, Any]) -> "PluginMetadata":
        known = set(cls.__dataclass_fields__)
        kw = {k: v for k, v in m.items() if k in known}
        kw["plugin_type"] = PluginType(m.get("plugin_type", "MODEL_COMPONENT"))
        kw.setdefault("version", "0.0.0")
        kw.setdefault("author", "")
        kw.setdefault("description", "")
        return cls(**kw)


class ModelPluginInterface:
    def __init__(self, metadata: PluginMetadata):
        self.metadata = metadata
        self._initialized = False

    @property
    def is_initialized(self) -> bool:
        return self._initialized

    def initialize(self, **kwargs) -> bool:
        self._initialized = True
        return True

    def cleanup(self) -> bool:
        self._initialized = False
        return True


class TextModelPluginInterface(ModelPluginInterface):
    def infer(self, data):
        raise NotImplementedError

    def generate_text(self, prompt, **kwargs):
        raise NotImplementedError

    def load_model(self, config=None):
        raise NotImplementedError

    def tokenize(self, text: str, **kwargs) -> List[int]:
        raise NotImplementedError

    def detokenize(self, token_ids: List[int], **kwargs) -> str:
        raise NotImplementedError

    def infer_batch(self, requests: List[Any]) -> List[Any]:
        """Default: serial loop (plugins override with the continuous batcher)."""
        return [self.generate_text(r) for r in requests]


class VisionLanguagePluginInterface(TextModelPluginInterface):
    """Text + image inputs: ``infer((text_or_ids, pixels))``."""

    def encode_images(self, images):
        raise NotImplementedError


class HardwareBackendInterface:
    """A compute backend a model can run on (``pio/plugins/base/gpu_interface.py:4-55``)."""

    name = "abstract"

    def initialize(self) -> bool:
        return True

    def get_device_info(self) -> Dict[str, Any]:
        return {}

    def allocate(self, nbytes: int):
        raise NotImplementedError

    def free(self, buf) -> None:
        pass

    def memcpy_h2d(self, dst, src) -> None:
        raise NotImplementedError

    def memcpy_d2h(self, dst, src) -> None:
        raise NotImplementedError

    def synchronize(self) -> None:
        pass

    def matmul(self, a, b):
        raise NotImplementedError

    def cleanup(self) -> None:
        pass
