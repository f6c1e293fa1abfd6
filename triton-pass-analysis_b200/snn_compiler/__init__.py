"""snn_compiler -- B200-native (sm_100a) multi-step SNN inference.

Drop-in for the reference's ``snn_compiler`` kernels and nn API
(Xarlley/Triton-Pass-Analysis, snn_compiler/__init__.py:1-39).  All device work
runs in libsnnb200.so: hand-written sm_100a CUDA kernels behind a C ABI
(include/snnb200.h), called through ctypes.  No Triton, no CPU fallback.
"""
from .kernels import (if_lif, plif, cuba_lif, eif, fused_bias_if_lif, fused_bias_if_lif_rate,
                      fused_bias_if_lif_stateful, fold_conv_bn, conv_neuron, linear_neuron,
                      conv_bn_neuron)
from .nn import (IFNode, LIFNode, PLIFNode, CubaLIFNode, EIFNode, FusedAddNeuron,
                 RateCodedIFNode, RateCodedLIFNode, StatefulLIFNode, FusedConvNeuron,
                 FusedLinearNeuron, FusedConvBNNeuron, FusedConvBNAddNeuron, ChunkedForward,
                 run_chunked)

__all__ = [
    "if_lif", "plif", "cuba_lif", "eif", "fused_bias_if_lif", "fused_bias_if_lif_rate",
    "fused_bias_if_lif_stateful", "fold_conv_bn", "conv_neuron", "linear_neuron",
    "conv_bn_neuron", "FusedConvNeuron", "FusedLinearNeuron", "FusedConvBNNeuron",
    "FusedConvBNAddNeuron",
    "IFNode", "LIFNode", "PLIFNode", "FusedAddNeuron", "RateCodedIFNode",
    "RateCodedLIFNode", "StatefulLIFNode", "CubaLIFNode", "EIFNode", "ChunkedForward",
    "run_chunked",
]
