"""Model zoo on the fused kernels (reference snn_compiler/zoo/)."""
from .vgg import (VGGSNN, SpikingVGG, random_vgg_params, vgg11_snn, vgg13_snn, vgg16_snn,
                  vgg19_snn, VGG16_CFG)
from .resnet import BasicBlockSNN, ResNetSNN, resnet18_snn, resnet34_snn
from .sew_resnet import SEWBasicBlockSNN, SEWResNetSNN, sew_resnet18_snn, sew_resnet34_snn

__all__ = ["VGGSNN", "SpikingVGG", "random_vgg_params", "vgg11_snn", "vgg13_snn", "vgg16_snn",
           "vgg19_snn", "VGG16_CFG", "BasicBlockSNN", "ResNetSNN", "resnet18_snn",
           "resnet34_snn", "SEWBasicBlockSNN", "SEWResNetSNN", "sew_resnet18_snn",
           "sew_resnet34_snn"]
