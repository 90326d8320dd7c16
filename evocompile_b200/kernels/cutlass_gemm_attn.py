"""Native-extension front of the catalog, backed by libgko_b200.so.

Drop-in for eval/kernels/cutlass_gemm_attn.py, which JIT-builds sm_80 CUTLASS /
WMMA extensions that cannot load on a B200. Here ``load_ext()`` returns the
already-built sm_100a library's operators under the reference's names
(``ext.fmha_fwd``, ``ext.addmm_epilogue``, ``ext.linear_swiglu``), and the
Python entry points keep their signatures:

* ``gko::cutlass_fmha_pair`` (:81-121) — same schema and autograd as
  gko::fused_sdpa_pair, same tcgen05 attention kernel;
* ``handwritten_attention`` (:124-178), ``can_handwritten`` (:69-75);
* ``addmm_epilogue(bias, mat1, mat2, act)`` (:181-186; act 0 none, 1 gelu, 2 relu);
* ``linear_swiglu_epilogue(x, weight)`` (:243-246).

A load or launch failure raises; there is no Triton fallback.
"""

from __future__ import annotations

import types
from typing import Tuple

import torch

from .. import _lib, ops

_OP = False


def load_ext():
    """The operators of the native library under the reference extension's names."""
    _lib.load()
    return types.SimpleNamespace(
        fmha_fwd=lambda q, k, v, bias, scale, causal, window, softcap: list(
            ops.fmha_fwd(q, k, v, bias, scale, causal, window, softcap)),
        addmm_epilogue=lambda bias, mat1, mat2, act: ops.addmm_act(bias, mat1, mat2, int(act)),
        linear_swiglu=ops.linear_swiglu,
    )


def load_swiglu_ext():
    return load_ext()


def can_handwritten(q):
    return q is not None and q.dim() == 4 and q.dtype in (torch.float16, torch.bfloat16) and int(q.size(-1)) in (64, 128)


def _ensure_op():
    global _OP
    if _OP:
        return
    if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "cutlass_fmha_pair")):

        @torch.library.custom_op("gko::cutlass_fmha_pair", mutates_args=())
        def cutlass_fmha_pair(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_bias: torch.Tensor,
                              scale: float, causal: int, window: int, softcap: float
                              ) -> Tuple[torch.Tensor, torch.Tensor]:
            return ops.fmha_fwd(q, k, v, attn_bias, scale, causal, window, softcap)

        @cutlass_fmha_pair.register_fake
        def _(q, k, v, attn_bias, scale, causal, window, softcap):
            return q.new_empty(q.shape), q.new_empty((q.size(0) * q.size(1), q.size(2)), dtype=torch.float32)

    from .fused_sdpa import _bwd_pair, _ensure_op as _ensure_sdpa, _setup_pair

    _ensure_sdpa()  # provides gko::fused_sdpa_bwd used by the backward
    try:
        torch.library.register_autograd("gko::cutlass_fmha_pair", _bwd_pair, setup_context=_setup_pair)
    except RuntimeError as e:
        if "already" not in str(e).lower() and "twice" not in str(e).lower():
            raise
    _OP = True


def handwritten_attention(q, k, v, attn_bias, scale, causal=0, window=0, softcap=0.0):
    """Fused attention through gko::cutlass_fmha_pair (shows up as a gko custom op in Inductor output)."""
    squeeze = q.dim() == 3
    if squeeze:
        q, k, v = q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)
    if attn_bias is None:
        attn_bias = q.new_empty((0,))
    _ensure_op()
    out, _ = torch.ops.gko.cutlass_fmha_pair(q, k, v, attn_bias, float(scale), int(causal), int(window or 0),
                                             float(softcap or 0.0))
    return out.squeeze(1) if squeeze else out


def addmm_epilogue(bias, mat1, mat2, act=1):
    """Tensor-core GEMM with a fused bias + activation epilogue. act: 0 none, 1 gelu, 2 relu."""
    return ops.addmm_act(bias, mat1, mat2, int(act))


def linear_swiglu_epilogue(x, weight):
    """x (..., D), weight (2H, D) -> silu(x Wg^T) * (x Wu^T), (..., H)."""
    return ops.linear_swiglu(x, weight)
