"""gko::gemm_swiglu — gate/up GEMM with the SwiGLU epilogue in one tcgen05 kernel.

Drop-in for eval/kernels/gemm_swiglu.py: ``torch.ops.gko.gemm_swiglu(x, weight)``
(schema :213-215) with x (..., D) and weight (2H, D) = [W_gate; W_up] returns
silu(x W_gate^T) * (x W_up^T) of shape (..., H) (fake :217-220). The [.., 2H]
intermediate never reaches memory. Autograd recomputes gate/up as the
reference's _backward (:177-200). ``apply(x, weight)`` is the public entry the
TorchTitan FusedSwiGLU hook calls (:244-250); ``swiglu_mlp`` adds the
down-projection on the same tensor-core GEMM.

Training form (no reference counterpart): ``torch.ops.gko.gemm_swiglu_aux(x, weight)
-> (out, gate_up)`` and ``apply_train(x, weight)``: the forward kernel also writes the
[.., 2H] gate/up pre-activations, the backward turns them into [d_gate | d_up] with one
elementwise kernel (gko_swiglu_bwd) and runs dX on the tensor-core GEMM, without the
reference backward's recomputation of the gate/up GEMM.
"""

from __future__ import annotations

from typing import Tuple

import torch

from .. import ops
from . import gemm_ops

_OP_READY = False
_AUTOGRADED = False
_PASS_INSTALLED = False


def gemm_swiglu(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """silu(x W_g^T) * (x W_u^T); x (..., D), weight (2H, D) -> (..., H)."""
    return ops.linear_swiglu(x, weight)


def _setup_context(ctx, inputs, output):
    x, weight = inputs
    ctx.save_for_backward(x, weight)


def _backward(ctx, grad_out):
    """The reference's backward (eval/kernels/gemm_swiglu.py:177-200): recompute gate/up, then
    dX and dW; every GEMM on the library's tensor-core kernel."""
    x, weight = ctx.saved_tensors
    x2 = x.reshape(-1, x.shape[-1])
    gate, up = torch.ops.gko.gemm(x2, weight.t()).chunk(2, dim=-1)
    g = grad_out.reshape(-1, grad_out.shape[-1])
    sig = torch.sigmoid(gate)
    d_up = g * gate * sig
    d_gate = g * up * (sig * (1 + gate * (1 - sig)))
    d_gu = torch.cat([d_gate, d_up], dim=-1)
    needs = getattr(ctx, "needs_input_grad", None) or (True, True)
    gx = torch.ops.gko.gemm(d_gu, weight).reshape(x.shape) if needs[0] else None
    gw = torch.ops.gko.gemm(d_gu.t(), x2) if needs[1] else None
    return gx, gw


def _setup_aux(ctx, inputs, output):
    x, weight = inputs
    ctx.save_for_backward(x, weight, output[1])


def _backward_aux(ctx, grad_out, grad_gu):
    x, weight, gate_up = ctx.saved_tensors
    d_gu = torch.ops.gko.swiglu_bwd(grad_out, gate_up)
    if grad_gu is not None:
        d_gu = d_gu + grad_gu
    needs = getattr(ctx, "needs_input_grad", None) or (True, True)
    d2 = d_gu.reshape(-1, d_gu.shape[-1])
    # dX = d_gate_up @ [Wg; Wu] on the tensor-core GEMM (the weight read as an MN-major operand)
    gx = torch.ops.gko.gemm(d2, weight).reshape(x.shape) if needs[0] else None
    # dW = d_gate_up^T @ X over the tokens: d_gate_up^T is read in place as an MN-major operand
    gw = torch.ops.gko.gemm(d2.t(), x.reshape(-1, x.shape[-1])) if needs[1] else None
    return gx, gw


def apply_train(x, weight):
    """silu(x Wg^T) * (x Wu^T) whose backward reuses the gate/up values saved by the forward kernel."""
    _ensure_op()
    return torch.ops.gko.gemm_swiglu_aux(x, weight)[0]


def _ensure_op():
    global _OP_READY, _AUTOGRADED
    gemm_ops.ensure()
    if not _OP_READY:
        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "gemm_swiglu")):

            @torch.library.custom_op("gko::gemm_swiglu", mutates_args=())
            def _op(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
                return gemm_swiglu(x, weight)

            @_op.register_fake
            def _(x, weight):
                return x.new_empty(*x.shape[:-1], weight.shape[0] // 2)

        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "gemm_swiglu_aux")):

            @torch.library.custom_op("gko::gemm_swiglu_aux", mutates_args=())
            def _aux(x: torch.Tensor, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
                return ops.linear_swiglu(x, weight, save_pre=True)

            @_aux.register_fake
            def _(x, weight):
                h = weight.shape[0] // 2
                return x.new_empty(*x.shape[:-1], h), x.new_empty(*x.shape[:-1], 2 * h)

            torch.library.register_autograd("gko::gemm_swiglu_aux", _backward_aux, setup_context=_setup_aux)

        _OP_READY = True
    if not _AUTOGRADED:
        try:
            torch.library.register_autograd("gko::gemm_swiglu", _backward, setup_context=_setup_context)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise
        _AUTOGRADED = True


def register(backend: str = "") -> None:
    """Install the custom op (no FX pass; callers hook FusedSwiGLU modules). ``backend`` is ignored."""
    global _PASS_INSTALLED
    _ensure_op()
    _PASS_INSTALLED = True


def apply(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Public entry for module hooks: the registered op (autograd-aware)."""
    _ensure_op()
    return torch.ops.gko.gemm_swiglu(x, weight)


def swiglu_mlp(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """Full SwiGLU MLP: gko::gemm_swiglu, then the down-projection h W_down^T."""
    return ops.linear(apply(x, w_gate_up), w_down)
