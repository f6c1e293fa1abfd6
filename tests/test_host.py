"""Host-side checks that need no GPU."""
import torch

from oracle import params as OP


def test_product_synthetic_weights_match_oracle_draws():
    """The engine's seeded VGG16 weights are bit-identical to the oracle's."""
    from snn_compiler.zoo.vgg import random_vgg_params
    a = random_vgg_params(1)
    b = OP.vgg16_params(1)
    assert len(a["convs"]) == len(b["convs"]) == 13
    for x, y in zip(a["convs"], b["convs"]):
        for k in ("w", "b", "gamma", "beta", "mean", "var"):
            assert torch.equal(x[k], y[k]), k
        assert x["pool"] == y["pool"]
    for x, y in zip(a["fcs"], b["fcs"]):
        assert torch.equal(x["w"], y["w"]) and torch.equal(x["b"], y["b"])


def test_fold_matches_oracle_fold():
    from snn_compiler.kernels.fused import fold_conv_bn
    from oracle import vgg as OV
    c = OP.vgg16_params(1)["convs"][3]
    w1, b1 = fold_conv_bn(c["w"], c["b"], c["gamma"], c["beta"], c["mean"], c["var"], c["eps"])
    w2, b2 = OV.fold_conv_bn(c["w"], c["b"], c["gamma"], c["beta"], c["mean"], c["var"], c["eps"])
    assert torch.equal(w1, w2) and torch.equal(b1, b2)


def test_vggsnn_module_structure_and_params():
    from snn_compiler.zoo.vgg import vgg16_snn
    m = vgg16_snn(num_classes=10, fc_in=512)
    P = m.params_dict()
    assert len(P["convs"]) == 13 and sum(c["pool"] for c in P["convs"]) == 5
    assert [tuple(f["w"].shape) for f in P["fcs"]] == [(4096, 512), (4096, 4096), (10, 4096)]
