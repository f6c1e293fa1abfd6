"""CPU oracle for the SNN multi-step inference hot path -- TEST INFRASTRUCTURE.

This package restates, on the CPU, the reference's own algorithms
(Xarlley/Triton-Pass-Analysis, ``snn_compiler/``) so that the CUDA kernels of
this repository can be checked against them on identical seeded inputs.  It is
the checker and the timed CPU baseline, never the thing measured or shipped:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import it.  The product path (``snn_compiler`` in ``triton-pass-analysis_b200/``)
never imports it and has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` ran the reference's own Python code
(naive_if_lif, fold_conv_bn, bitpack_N, VGGSNN.forward, the reference test
suite's _RefSSA block) on seeded inputs and committed the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against
them.  PLIF has no counterpart in the reference (it is SpikingJelly's
ParametricLIFNode) and is pinned only through its k=0.5 identity with LIF tau=2.

Modules:
  neurons    -- multi-step IF/LIF/PLIF (C core in lif.c, built to _build/liboracle.so)
  bitops     -- bit packing and the {0,1}x{+-1} / {0,1}x{0,1} popcount GEMMs
  vgg        -- VGG16-SNN (conv + BN + LIF + maxpool, classifier) parameters and forward
  attention  -- spiking self-attention block (Q/K/V projections, K^T V, A V + LIF)
  params     -- seeded synthetic inputs and weights with the benchmark distributions
"""
