"""B200-native (sm_100a) fused operators with the torch.ops.gko interface of
EvoCompile's kernel catalog: GEMM+bias+GELU, GEMM+SwiGLU (+ down-projection)
and fused multi-head attention forward (causal, GQA, varlen).

The CUDA kernels and their C ABI live in libgko_b200.so (built by
``python -m evocompile_b200.build``); ``evocompile_b200.kernels`` mirrors the
reference's ``eval/kernels`` package (catalog, register(), FX passes).
"""

__version__ = "0.1.0"

from . import ops  # noqa: F401,E402
