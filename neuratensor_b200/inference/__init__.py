from .engine import InferenceEngine, InferenceResult

__all__ = ["InferenceEngine", "InferenceResult"]
