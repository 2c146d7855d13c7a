"""B200-native (sm_100a) fused DeepSeek-V3 FP8 block-scale MoE layer.

``kernelforge_b200.kernel`` is a drop-in for the reference operator
``solution/triton/kernel.py::kernel``; the compute runs in ``libkf_moe.so``.
"""
from .binding import experts, kernel, route  # noqa: F401
