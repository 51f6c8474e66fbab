"""Model implementations (dense, MoE, MLA, hybrid) and weight sources."""
from .presets import PRESETS, get_preset  # noqa: F401
from .registry import get_model_class, register_model, supported_architectures  # noqa: F401
