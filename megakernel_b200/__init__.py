"""B200-native persistent decode megakernel for Qwen3-0.6B-shaped decoders.

The compute path is libmegakernel.so (hand-written CUDA for sm_100a, C ABI in
include/megakernel.h); this package holds the host glue around it.
"""
from .shapes import SHAPES, QWEN3_0_6B_D64, QWEN3_0_6B_D128, TINY, Shape  # noqa: F401
