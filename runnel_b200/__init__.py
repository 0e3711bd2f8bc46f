"""runnel-b200: Runnel's Ornith sparse-MoE block hot path on NVIDIA B200.

The kernels live in ``librnb_moe.so`` (C ABI in include/rnb_moe.h, CUDA
sources in runnel_b200/csrc).  Python modules mirror the reference's
operator interface:

* :mod:`runnel_b200.mlx` -- ``fuse_routed_gate_up(model)`` and the packed
  ``FusedQuantizedSwitchGLU`` (src/runnel/mlx.py in the reference);
* :mod:`runnel_b200.switch_layers` -- SwitchGLU / shared expert /
  ``SparseMoeBlock`` modules with mlx-lm's names and signatures;
* :mod:`runnel_b200.ops` -- functional calls on device tensors;
* :mod:`runnel_b200.inputs` -- seeded synthetic blocks for tests and benchmarks.
"""
__version__ = "0.1.0"
