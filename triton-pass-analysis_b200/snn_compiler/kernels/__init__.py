"""Kernel entry points (reference snn_compiler/kernels/__init__.py), backed by libsnnb200.so."""
from .neurons import if_lif, plif, cuba_lif, eif, neuron_multistep
from .fused import (fused_bias_if_lif, fused_bias_if_lif_rate, fused_bias_if_lif_stateful,
                    fold_conv_bn, conv_neuron, linear_neuron, conv_bn_neuron)

__all__ = [
    "if_lif", "plif", "cuba_lif", "eif", "neuron_multistep",
    "fused_bias_if_lif", "fused_bias_if_lif_rate", "fused_bias_if_lif_stateful",
    "fold_conv_bn", "conv_neuron", "linear_neuron", "conv_bn_neuron",
]
