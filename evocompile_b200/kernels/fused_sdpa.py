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

Additions over the reference Triton path: GQA (k/v with H/g heads) and varlen.
Supported: float16/bfloat16, D in {64, 128}; anything else raises (there is no
eager fallback). The backward currently recomputes attention with ATen in
fp32 from the saved lse (the reference's recompute formulation).
"""

from __future__ import annotations

from typing import Tuple

import torch

from .. import ops

_OP_READY = False
_AUTOGRADED = False


# --------------------------------------------------------------------------- backward (ATen recompute)
def _softcap_tanh(s, softcap):
    x = torch.clamp(s / softcap, -15.0, 15.0)
    return softcap * torch.tanh(x), x


def _attention_bwd(q, k, v, attn_bias, out, lse, dout, scale, causal, window, softcap):
    """dq, dk, dv of softmax(mask(softcap(scale q k^T + bias))) v, from the saved lse.

    Processes one batch entry at a time so the [H, Sq, Sk] score block stays bounded.
    """
    z, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    g = hq // hkv
    dq = torch.empty_like(q, memory_format=torch.contiguous_format)
    dk = torch.zeros(k.shape, device=k.device, dtype=torch.float32)
    dv = torch.zeros(v.shape, device=v.device, dtype=torch.float32)
    bias_t, mode, bstr, nb = ops._bias_layout(q, k, attn_bias)
    qi = torch.arange(sq, device=q.device)[:, None]
    ki = torch.arange(sk, device=q.device)[None, :]
    keep = torch.ones(sq, sk, dtype=torch.bool, device=q.device)
    if causal:
        keep &= ki <= qi
    if window and window > 0:
        keep &= (ki - qi <= window) & (qi - ki <= window)
    lse4 = lse.view(z, hq, sq, 1)
    for b in range(z):
        qb = q[b].float()
        kb = k[b].float().repeat_interleave(g, dim=0)
        vb = v[b].float().repeat_interleave(g, dim=0)
        s = torch.matmul(qb, kb.transpose(-1, -2)) * scale
        if mode != 0:
            bb = _dense_bias(bias_t, mode, bstr, nb, b, hq, sq, sk)
            s = s + bb
        x = None
        if softcap and softcap > 0:
            s, x = _softcap_tanh(s, softcap)
        s = s.masked_fill(~keep, float("-inf"))
        l = lse4[b]
        p = torch.exp(s - torch.where(torch.isinf(l), torch.zeros_like(l), l))
        p = torch.where(torch.isinf(l), torch.zeros_like(p), p)
        do = dout[b].float()
        dvb = torch.matmul(p.transpose(-1, -2), do)
        dp = torch.matmul(do, vb.transpose(-1, -2))
        delta = (do * out[b].float()).sum(-1, keepdim=True)
        ds = p * (dp - delta)
        if x is not None:
            ds = ds * (1 - torch.tanh(x) ** 2) * ((x > -15.0) & (x < 15.0))
        dq[b] = (torch.matmul(ds, kb) * scale).to(q.dtype)
        dkb = torch.matmul(ds.transpose(-1, -2), qb) * scale
        dk[b] += dkb.view(hkv, g, sk, d).sum(1)
        dv[b] += dvb.view(hkv, g, sk, d).sum(1)
    return dq, dk.to(k.dtype), dv.to(v.dtype)


def _dense_bias(bias_t, mode, bstr, nb, b, h, sq, sk):
    bi = b % nb
    if mode == 1:  # key padding
        row = torch.as_strided(bias_t, (sk,), (bstr[3],), bias_t.storage_offset() + bi * bstr[0])
        return row.float().view(1, 1, sk)
    full = torch.as_strided(bias_t, (h, sq, sk), (bstr[1], bstr[2], bstr[3]), bias_t.storage_offset() + bi * bstr[0])
    return full.float()


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
                return _attention_bwd(q, k, v, attn_bias, out, lse, dout, scale, causal, window, softcap)

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
