"""Cortex model family (drop-in for the reference's ``cortex.models``)."""

from cortex.models.config import CORTEX_M, CORTEX_S, CORTEX_XS, CortexConfig
from cortex.models.cortex import BehaviorDecoder, CortexModel, MaskedSpikeHead
from cortex.models.perceiver import CrossAttentionBlock, PerceiverEncoder, SelfAttentionBlock
from cortex.models.tokenizer import SpikeTokenizer

__all__ = [
    "CORTEX_M", "CORTEX_S", "CORTEX_XS", "BehaviorDecoder", "CortexConfig", "CortexModel",
    "CrossAttentionBlock", "MaskedSpikeHead", "PerceiverEncoder", "SelfAttentionBlock",
    "SpikeTokenizer",
]
