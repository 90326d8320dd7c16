"""gko::gemm_swiglu — gate/up GEMM with the SwiGLU epilogue in one tcgen05 kernel.

Drop-in for eval/kernels/gemm_swiglu.py: ``torch.ops.gko.gemm_swiglu(x, weight)``
(schema :213-215) with x (..., D) and weight (2H, D) = [W_gate; W_up] returns
silu(x W_gate^T) * (x W_up^T) of shape (..., H) (fake :217-220). The [.., 2H]
intermediate never reaches memory. Autograd recomputes gate/up as the
reference's _backward (:177-200). ``apply(x, weight)`` is the public entry the
TorchTitan FusedSwiGLU hook calls (:244-250); ``swiglu_mlp`` adds the
down-projection on the same tensor-core GEMM.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops

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
    x, weight = ctx.saved_tensors
    gate, up = F.linear(x, weight).chunk(2, dim=-1)
    sig = torch.sigmoid(gate)
    d_up = grad_out * gate * sig
    d_gate = grad_out * up * (sig * (1 + gate * (1 - sig)))
    d_gu = torch.cat([d_gate, d_up], dim=-1)
    needs = getattr(ctx, "needs_input_grad", None) or (True, True)
    gx = F.linear(d_gu, weight.t()).reshape(x.shape) if needs[0] else None
    gw = None
    if needs[1]:
        gw = d_gu.reshape(-1, d_gu.shape[-1]).t().mm(x.reshape(-1, x.shape[-1]))
    return gx, gw


def _ensure_op():
    global _OP_READY, _AUTOGRADED
    if not _OP_READY:
        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "gemm_swiglu")):

            @torch.library.custom_op("gko::gemm_swiglu", mutates_args=())
            def _op(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
                return gemm_swiglu(x, weight)

            @_op.register_fake
            def _(x, weight):
                return x.new_empty(*x.shape[:-1], weight.shape[0] // 2)

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
