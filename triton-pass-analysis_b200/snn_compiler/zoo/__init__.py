"""Model zoo on the fused kernels (reference snn_compiler/zoo/)."""
from .vgg import (VGGSNN, SpikingVGG, random_vgg_params, vgg11_snn, vgg13_snn, vgg16_snn,
                  vgg19_snn, VGG16_CFG)

__all__ = ["VGGSNN", "SpikingVGG", "random_vgg_params", "vgg11_snn", "vgg13_snn", "vgg16_snn",
           "vgg19_snn", "VGG16_CFG"]
