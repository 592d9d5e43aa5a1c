"""neuratensor_b200 -- NeuraTensor's FusedSpikeBlock inference path on B200 (sm_100a) kernels.

The public names mirror the reference package ``neuratensor`` 4.0.4 (model,
layers, presets, engine, backend detection); the block hot path runs in
``lib/libneuratensor_native.so`` through the C ABI in
``include/neuratensor_native.h``.  See ``neuratensor_b200.backends`` for
the switch that routes an installed ``neuratensor`` through the same kernels.
"""
__version__ = "0.1.0"
REFERENCE_VERSION = "4.0.4"

from .core.model import NeuraTensorModel, ModelConfig, SlidingWindowAttention, RotaryEmbedding
from .core.snn import LIFLayer, AdaptiveLIFLayer
from .core.ssm import SelectiveSSMLayer, SSMLayer
from .core.fused import FusedSpikeBlock, FusedSNNSSMBlock, BlockState
from .config.presets import get_preset, list_presets, PRESETS
from .inference.engine import InferenceEngine, InferenceResult
from .backends.detect import detect_backend

NeuraTensor = NeuraTensorModel

__all__ = ["NeuraTensor", "NeuraTensorModel", "ModelConfig", "LIFLayer", "AdaptiveLIFLayer", "SelectiveSSMLayer",
           "SSMLayer", "FusedSpikeBlock", "FusedSNNSSMBlock", "BlockState", "SlidingWindowAttention",
           "RotaryEmbedding", "get_preset", "list_presets", "PRESETS", "InferenceEngine", "InferenceResult",
           "detect_backend", "__version__"]
