"""nn.Module API (reference snn_compiler/nn/__init__.py)."""
from .modules import (IFNode, LIFNode, PLIFNode, CubaLIFNode, EIFNode, FusedAddNeuron,
                      RateCodedIFNode, RateCodedLIFNode, StatefulLIFNode)
from .chunked import ChunkedForward, run_chunked
from .fused_layers import (FusedConvNeuron, FusedLinearNeuron, FusedConvBNNeuron,
                           FusedConvBNAddNeuron, FusedConvBN, tune_convs)
from .attention import (FusedSpikeAttention, SpikeAttentionBlock, is_spiking_self_attention,
                        is_ms_attention, is_spiking_attention)

__all__ = ["IFNode", "LIFNode", "PLIFNode", "CubaLIFNode", "EIFNode", "ChunkedForward",
           "run_chunked", "FusedAddNeuron", "FusedConvNeuron",
           "FusedLinearNeuron", "FusedConvBNNeuron", "FusedConvBNAddNeuron", "FusedConvBN", "tune_convs", "RateCodedIFNode",
           "RateCodedLIFNode", "StatefulLIFNode", "FusedSpikeAttention", "SpikeAttentionBlock",
           "is_spiking_self_attention", "is_ms_attention", "is_spiking_attention"]
