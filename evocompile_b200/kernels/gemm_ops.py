"""Opaque operators for the GEMMs inside the backward formulas of gko::addmm_gelu and
gko::gemm_swiglu (no reference counterpart: the reference's backward calls torch.mm / F.linear).

AOTAutograd traces a registered backward formula under torch.compile, so the formula may only
call torch operators or opaque custom ops; these wrap the library's tensor-core GEMM and the
SwiGLU backward kernel so that a compiled training step still runs them as single launches.

``torch.ops.gko.gemm(mat1, mat2)``: mat1 [m, k] @ mat2 [k, n] on the tcgen05 GEMM. A transposed
mat1 (the weight gradient dZ^T X) and a transposed mat2 (a Linear weight's W^T view) are read in
place. ``torch.ops.gko.swiglu_bwd(dy, gate_up)``: [d_gate | d_up] of silu(g) * u.
"""

from __future__ import annotations

import torch

from .. import _lib, ops

_READY = False


def ensure() -> None:
    """Define the ops once per process (idempotent)."""
    global _READY
    if _READY:
        return
    if not hasattr(torch.ops.gko, "gemm"):

        @torch.library.custom_op("gko::gemm", mutates_args=())
        def _gemm(mat1: torch.Tensor, mat2: torch.Tensor) -> torch.Tensor:
            return ops.addmm_act(None, mat1, mat2, _lib.ACT_NONE)

        @_gemm.register_fake
        def _(mat1, mat2):
            return mat1.new_empty(mat1.shape[0], mat2.shape[1])

    if not hasattr(torch.ops.gko, "swiglu_bwd"):

        @torch.library.custom_op("gko::swiglu_bwd", mutates_args=())
        def _swiglu_bwd(dy: torch.Tensor, gate_up: torch.Tensor) -> torch.Tensor:
            return ops.swiglu_bwd(dy.contiguous(), gate_up)

        @_swiglu_bwd.register_fake
        def _(dy, gate_up):
            return gate_up.new_empty(gate_up.shape)

    _READY = True
