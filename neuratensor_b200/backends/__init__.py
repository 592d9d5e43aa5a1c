from .detect import BackendInfo, detect_backend
from .native import native_available, use_native, patch_reference

__all__ = ["BackendInfo", "detect_backend", "native_available", "use_native", "patch_reference"]
