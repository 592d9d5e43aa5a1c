from .snn import LIFLayer, AdaptiveLIFLayer
from .ssm import SelectiveSSMLayer, SSMLayer
from .fused import FusedSpikeBlock, FusedSNNSSMBlock, BlockState
from .model import NeuraTensorModel, NeuraTensor, ModelConfig, SlidingWindowAttention, RotaryEmbedding

__all__ = ["LIFLayer", "AdaptiveLIFLayer", "SelectiveSSMLayer", "SSMLayer", "FusedSpikeBlock", "FusedSNNSSMBlock",
           "BlockState", "NeuraTensorModel", "NeuraTensor", "ModelConfig", "SlidingWindowAttention",
           "RotaryEmbedding"]
