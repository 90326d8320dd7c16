"""Fused attention ops on the tcgen05 FMHA forward kernel.

Drop-in for eval/kernels/fused_sdpa.py:

* ``fused_attention(q, k, v, attn_bias, scale, causal=0, window=0, softcap=0.0)``
  — the hook target of the attention rewrites (:796-840). q/k/v are
  [Z, H, S, D] (any strides with unit stride along D, read in place — no
  ``.contiguous()`` copy of [B, S, H, D]-derived views) or 3-D [Z, S, D].
* ``torch.ops.gko.fused_sdpa_pair(q, k, v, attn_bias, scale, causal, window,
  softcap) -> (out, lse)`` (:912-943): out is a fresh dense [Z, H, Sq, D]
  tensor, lse fp32 [Z*H, Sq] = rowmax + ln(rowsum).
* ``torch.ops.gko.fused_sdpa_bwd(...) -> (dq, dk, dv)`` (:947-967) and
  ``torch.ops.gko.fused_sdpa(q, k, v, attn_bias, scale, causal)`` (:981-994)
  with the autograd wiring of :843-898.
* ``torch.ops.gko.fmha_varlen_fwd`` — packed variable-length sequences with
  GQA (no reference counterpart).

* ``torch.ops.gko.fmha_varlen_bwd`` — its backward (autograd of
  ``fmha_varlen_fwd`` is registered).

Additions over the reference Triton path: GQA (k/v with H/g heads) and varlen.
Supported: float16/bfloat16, D in {64, 128}; anything else raises (there is no
eager fallback). The backward is the library's tcgen05 kernel (gko_fmha_bwd):
it recomputes P from the saved lse, as the reference's Triton backward does.
"""

from __future__ import annotations

from typing import Tuple

import torch

from .. import ops

_OP_READY = False
_AUTOGRADED = False


# --------------------------------------------------------------------------- python entry points
def fused_sdpa_forward(q, k, v, attn_bias, scale, causal=0):
    return ops.fmha_fwd(q, k, v, attn_bias, float(scale), int(causal))[0]


def fused_attention(q, k, v, attn_bias, scale, causal=0, window=0, softcap=0.0):
    """Differentiable fused attention; Dynamo-safe (calls the custom op)."""
    squeeze = q.dim() == 3
    if squeeze:
        q, k, v = q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)
    if attn_bias is None:
        attn_bias = q.new_empty((0,))
    _ensure_op()
    out, _ = torch.ops.gko.fused_sdpa_pair(q, k, v, attn_bias, float(scale), int(causal), int(window or 0),
                                           float(softcap or 0.0))
    return out.squeeze(1) if squeeze else out


def _setup_pair(ctx, inputs, output):
    q, k, v, attn_bias, scale, causal, window, softcap = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, attn_bias, out, lse)
    ctx.scale, ctx.causal, ctx.window, ctx.softcap = float(scale), int(causal), int(window), float(softcap)


def _bwd_pair(ctx, dout, dlse):
    q, k, v, attn_bias, out, lse = ctx.saved_tensors
    dq, dk, dv = torch.ops.gko.fused_sdpa_bwd(q, k, v, attn_bias, out, lse, dout, ctx.scale, ctx.causal,
                                               ctx.window, ctx.softcap)
    return dq, dk, dv, None, None, None, None, None


def _setup_context(ctx, inputs, output):
    q, k, v, attn_bias, scale, causal = inputs
    ctx.save_for_backward(q, k, v, attn_bias, output)
    ctx.scale, ctx.causal = float(scale), int(causal)


def _backward(ctx, grad_out):
    q, k, v, attn_bias, out = ctx.saved_tensors
    _, lse = ops.fmha_fwd(q, k, v, attn_bias, ctx.scale, ctx.causal)
    dq, dk, dv = torch.ops.gko.fused_sdpa_bwd(q, k, v, attn_bias, out, lse, grad_out, ctx.scale, ctx.causal, 0, 0.0)
    return dq, dk, dv, None, None, None


def _setup_varlen(ctx, inputs, output):
    q, k, v, cu_q, cu_k, max_q, max_k, scale, causal = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse, cu_q, cu_k)
    ctx.max_q, ctx.max_k, ctx.scale, ctx.causal = int(max_q), int(max_k), float(scale), int(causal)


def _varlen_bwd(ctx, dout, dlse):
    q, k, v, out, lse, cu_q, cu_k = ctx.saved_tensors
    dq, dk, dv = torch.ops.gko.fmha_varlen_bwd(q, k, v, out, lse, dout, cu_q, cu_k, ctx.max_q, ctx.max_k,
                                               ctx.scale, ctx.causal)
    return dq, dk, dv, None, None, None, None, None, None


def _ensure_op():
    global _OP_READY, _AUTOGRADED
    if not _OP_READY:
        have = lambda n: hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, n)  # noqa: E731
        if not have("fused_sdpa_pair"):

            @torch.library.custom_op("gko::fused_sdpa_pair", mutates_args=())
            def fused_sdpa_pair(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_bias: torch.Tensor,
                                scale: float, causal: int, window: int, softcap: float
                                ) -> Tuple[torch.Tensor, torch.Tensor]:
                return ops.fmha_fwd(q, k, v, attn_bias, scale, causal, window, softcap)

            @fused_sdpa_pair.register_fake
            def _(q, k, v, attn_bias, scale, causal, window, softcap):
                # dense outputs: the kernel never returns q's (possibly transposed) strides
                return q.new_empty(q.shape), q.new_empty((q.size(0) * q.size(1), q.size(2)), dtype=torch.float32)

        if not have("fused_sdpa_bwd"):

            @torch.library.custom_op("gko::fused_sdpa_bwd", mutates_args=())
            def fused_sdpa_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_bias: torch.Tensor,
                               out: torch.Tensor, lse: torch.Tensor, dout: torch.Tensor, scale: float, causal: int,
                               window: int, softcap: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
                return ops.fmha_bwd(q, k, v, attn_bias, out, lse, dout, scale, causal, window, softcap)

            @fused_sdpa_bwd.register_fake
            def _(q, k, v, attn_bias, out, lse, dout, scale, causal, window, softcap):
                return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)

        try:
            torch.library.register_autograd("gko::fused_sdpa_pair", _bwd_pair, setup_context=_setup_pair)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise

        if not have("fused_sdpa"):

            @torch.library.custom_op("gko::fused_sdpa", mutates_args=())
            def fused_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_bias: torch.Tensor,
                           scale: float, causal: int) -> torch.Tensor:
                return fused_sdpa_forward(q, k, v, attn_bias, scale, causal)

            @fused_sdpa.register_fake
            def _(q, k, v, attn_bias, scale, causal):
                return q.new_empty(q.shape)

        if not have("fmha_varlen_fwd"):

            @torch.library.custom_op("gko::fmha_varlen_fwd", mutates_args=())
            def fmha_varlen_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                                cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, scale: float,
                                causal: int) -> Tuple[torch.Tensor, torch.Tensor]:
                return ops.fmha_varlen_fwd(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                           scale, causal)

            @fmha_varlen_fwd.register_fake
            def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, scale, causal):
                return q.new_empty(q.shape), q.new_empty((q.size(1), q.size(0)), dtype=torch.float32)

        if not have("fmha_varlen_bwd"):

            @torch.library.custom_op("gko::fmha_varlen_bwd", mutates_args=())
            def fmha_varlen_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                                lse: torch.Tensor, dout: torch.Tensor, cu_seqlens_q: torch.Tensor,
                                cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, scale: float,
                                causal: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
                return ops.fmha_varlen_bwd(q, k, v, out, lse, dout, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                           max_seqlen_k, scale, causal)

            @fmha_varlen_bwd.register_fake
            def _(q, k, v, out, lse, dout, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, scale, causal):
                return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)

        try:
            torch.library.register_autograd("gko::fmha_varlen_fwd", _varlen_bwd, setup_context=_setup_varlen)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise

        _OP_READY = True
    if not _AUTOGRADED:
        try:
            torch.library.register_autograd("gko::fused_sdpa", _backward, setup_context=_setup_context)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise
        _AUTOGRADED = True


def register(backend=None):
    """Install the attention ops. ``backend`` (triton/cutlass/auto/...) is accepted and ignored."""
    _ensure_op()


# --------------------------------------------------------------------------- microbenchmark
def microbench(*, z=128, h=12, s=128, d=64, dtype=torch.float16, warmup=10, iters=50, train=False, causal=0):
    """Time unfused bmm+softmax, in-tree SDPA and the fused op; report max-abs error vs unfused
    (the comparison of the reference's microbench, eval/kernels/fused_sdpa.py:1050-1133)."""
    register()
    dev = "cuda"
    scale = d ** -0.5
    bias = torch.zeros(z, s, device=dev, dtype=dtype)

    def make():
        ts = [torch.randn(z, h, s, d, device=dev, dtype=dtype) for _ in range(3)]
        return [t.requires_grad_(train) for t in ts]

    def unfused(q, k, v):
        sc = torch.matmul(q, k.transpose(-1, -2)) * scale
        if causal:
            idx = torch.arange(s, device=q.device)
            sc = sc.masked_fill(idx[None, None, None, :] > idx[None, None, :, None], -65504.0)
        return torch.matmul(torch.softmax(sc.float(), dim=-1).to(q.dtype), v)

    def sdpa(q, k, v):
        return torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale, is_causal=bool(causal))

    def fused(q, k, v):
        return fused_attention(q, k, v, bias, float(scale), int(causal))

    def timed(fn):
        q, k, v = make()

        def step():
            if train:
                for t in (q, k, v):
                    t.grad = None
                fn(q, k, v).square().mean().backward()
            else:
                fn(q, k, v)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            step()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    res = {name: timed(fn) for name, fn in (("unfused_bmm", unfused), ("in_tree_sdpa", sdpa), ("gko_fused", fused))}
    q0, k0, v0 = [t.detach() for t in make()]
    with torch.no_grad():
        ref = unfused(q0, k0, v0)
        res["gko_max_abs"] = float((fused(q0, k0, v0) - ref).abs().max())
        res["sdpa_max_abs"] = float((sdpa(q0, k0, v0) - ref).abs().max())
    res["train"], res["causal"] = int(train), int(causal)
    return res
