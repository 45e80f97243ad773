from .models import ModelConfig, VisionConfig, VLConfig, from_hf_dict, load_config  # noqa: F401
from .presets import PRESETS, get_preset  # noqa: F401
