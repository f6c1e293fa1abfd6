"""nn.Module API (reference snn_compiler/nn/__init__.py)."""
from .modules import (IFNode, LIFNode, PLIFNode, FusedAddNeuron, RateCodedIFNode,
                      RateCodedLIFNode, StatefulLIFNode)

__all__ = ["IFNode", "LIFNode", "PLIFNode", "FusedAddNeuron", "RateCodedIFNode",
           "RateCodedLIFNode", "StatefulLIFNode"]
