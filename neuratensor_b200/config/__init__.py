from .presets import PRESETS, get_preset, list_presets

__all__ = ["PRESETS", "get_preset", "list_presets"]
