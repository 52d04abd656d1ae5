"""Model definitions: the OLMo decoder and its building blocks."""
from .blocks import OLMoBlock, OLMoBlockGroup, OLMoLlamaBlock, OLMoSequentialBlock
from .layers import (
    Activation,
    BufferCache,
    Dropout,
    GELU,
    LayerNorm,
    LayerNormBase,
    ReLU,
    RMSLayerNorm,
    RotaryEmbedding,
    SwiGLU,
)
from .olmo import OLMo, OLMoGenerateOutput, OLMoOutput

__all__ = [
    "OLMo", "OLMoOutput", "OLMoGenerateOutput", "OLMoBlock", "OLMoSequentialBlock", "OLMoLlamaBlock",
    "OLMoBlockGroup", "LayerNormBase", "LayerNorm", "RMSLayerNorm", "RotaryEmbedding", "Activation",
    "GELU", "ReLU", "SwiGLU", "BufferCache", "Dropout",
]
