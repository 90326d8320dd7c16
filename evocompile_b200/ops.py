"""Tensor-level host code for the fused operators: validates torch tensors,
allocates outputs, and calls the C ABI of libgko_b200.so on the current stream.

These functions are what the ``gko::`` custom ops (``evocompile_b200.kernels``)
run. Each raises RuntimeError for inputs the kernels do not implement; none of
them falls back to another implementation.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_I64x4 = ctypes.c_int64 * 4


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _status_ptr(dev):
    return ctypes.c_void_p(_lib.status_word(dev).data_ptr())


def _stream(dev):
    return ctypes.c_void_p(_lib.stream_ptr(dev))


def _byte_range(t):
    """[first, last) byte addresses a tensor's elements can touch (empty tensors touch none)."""
    if t.numel() == 0:
        return (0, 0)
    lo = hi = t.data_ptr()
    for size, stride in zip(t.shape, t.stride()):
        span = (size - 1) * stride * t.element_size()
        if span < 0:
            lo += span
        else:
            hi += span
    return (lo, hi + t.element_size())


def _check_no_overlap(name, out, **operands):
    """Raise if ``out`` shares memory with an operand the kernel reads while it writes ``out``:
    epilogue stores of one CTA would race with another CTA's TMA loads of that operand."""
    o_lo, o_hi = _byte_range(out)
    for arg, t in operands.items():
        if t is None:
            continue
        lo, hi = _byte_range(t)
        if lo < o_hi and o_lo < hi:
            raise RuntimeError(f"{name}: out overlaps {arg} (the GEMM would read {arg} while writing out)")


# --------------------------------------------------------------------------- GEMM
def set_gemm_ctas(ctas: int) -> int:
    """Cap the SMs every tensor-core GEMM launched afterwards occupies (0: all); returns the
    previous cap. Leaves SMs to a collective running on another stream (gko_set_gemm_ctas)."""
    prev = _lib.load().gko_set_gemm_ctas(int(ctas))
    if prev < 0:
        _lib.check(_lib.ERR_INVALID, "gko_set_gemm_ctas")
    return prev


def addmm_act(bias, mat1, mat2, act: int = _lib.ACT_GELU, save_pre: bool = False, out=None):
    """act(mat1 @ mat2 + bias) with mat1 [..., K] and mat2 [K, N].

    Follows the contract of gko::addmm_gelu (eval/kernels/addmm_gelu.py:150-161,
    192-210): output shape mat1.shape[:-1] + (N,), dtype of mat1. mat2 is
    usually the transposed view W^T of a Linear weight and is read in place.
    With save_pre, returns (out, z) where z = mat1 @ mat2 + bias is written by the same
    kernel (bf16 / f16), for a backward that needs no recomputation.
    """
    dev = _lib.require_cuda(mat1, mat2, bias)
    if mat2.dim() != 2:
        raise RuntimeError(f"addmm_gelu: mat2 must be 2-D, got shape {tuple(mat2.shape)}")
    if mat1.dim() < 1:
        raise RuntimeError("addmm_gelu: mat1 must have at least one dimension")
    if mat1.dtype != mat2.dtype:
        raise RuntimeError(f"addmm_gelu: mat1 {mat1.dtype} and mat2 {mat2.dtype} differ")
    K = mat1.shape[-1]
    if mat2.shape[0] != K:
        raise RuntimeError(f"addmm_gelu: K mismatch {K} vs {mat2.shape[0]}")
    N = mat2.shape[1]
    dt = _lib.dtype_code(mat1.dtype)
    lead = mat1.shape[:-1]
    a = mat1.reshape(-1, K) if mat1.dim() != 2 else mat1
    M = a.shape[0]
    # a transposed mat1 (the weight-gradient GEMM dZ^T X) is read in place as an MN-major operand
    # when no activation or pre-activation output is asked for; other strides are made row-major
    a_mn = (dt != _lib.F32 and act == _lib.ACT_NONE and not save_pre and M > 1
            and a.stride(0) == 1 and (K == 1 or a.stride(1) % 8 == 0))
    if dt != _lib.F32 and a.stride(-1) != 1 and M > 1 and not a_mn:
        a = a.contiguous()
    b = mat2
    if dt != _lib.F32 and not (b.stride(0) == 1 or b.stride(1) == 1):
        b = b.contiguous()
    bias_t = None
    bias_dt = 0
    if bias is not None and bias.numel() > 0:
        if bias.numel() == N:
            bias_t = bias.reshape(N)
        elif bias.numel() == 1:
            bias_t = bias.reshape(1).expand(N)
        else:
            raise RuntimeError(
                f"addmm_gelu: bias must broadcast along rows (numel N={N}); got shape {tuple(bias.shape)}"
            )
        if bias_t.stride(0) != 1:
            bias_t = bias_t.contiguous()
        if bias_t.data_ptr() % 16:
            bias_t = bias_t.clone()  # the tensor-core epilogue reads the bias with 16-byte loads
        bias_dt = _lib.dtype_code(bias_t.dtype)
    if out is None:
        out = torch.empty((M, N), device=dev, dtype=mat1.dtype)
    elif mat1.dim() != 2 or tuple(out.shape) != (M, N) or out.dtype != mat1.dtype or out.stride(1) != 1:
        raise RuntimeError("addmm_act: out must be a row-major [m, n] tensor of mat1's dtype (2-D mat1)")
    else:
        _check_no_overlap("addmm_act", out, mat1=mat1, mat2=mat2)
    z = torch.empty((M, N), device=dev, dtype=mat1.dtype) if save_pre else None
    if M and N:
        with torch.cuda.device(dev):
            a_sm = a.stride(0) if M > 1 else max(K, 8)
            a_sk = a.stride(1)
            if a_mn and K == 1:
                a_sk = (M + 7) // 8 * 8  # a single row of the [K, M] storage: its stride is never used
            if save_pre:
                rc = _lib.load().gko_addmm_act_aux(
                    dt, act, M, N, K, _ptr(a), a_sm, a.stride(1), _ptr(b), b.stride(0), b.stride(1),
                    _ptr(bias_t), bias_dt, _ptr(out), out.stride(0), _ptr(z), z.stride(0), _status_ptr(dev),
                    _stream(dev),
                )
            else:
                rc = _lib.load().gko_addmm_act(
                    dt, act, M, N, K, _ptr(a), a_sm, a_sk, _ptr(b), b.stride(0), b.stride(1),
                    _ptr(bias_t), bias_dt, _ptr(out), out.stride(0), _status_ptr(dev), _stream(dev),
                )
        _lib.check(rc, "gko_addmm_act_aux" if save_pre else "gko_addmm_act")
    if save_pre:
        return out.reshape(*lead, N), z.reshape(*lead, N)
    return out.reshape(*lead, N)


def linear(x, weight, bias=None, out=None):
    """x @ weight.T (+ bias) on the tensor-core GEMM (the down-projection path); ``out`` (2-D x
    only) receives the result in place of a new tensor."""
    return addmm_act(bias, x, weight.t(), _lib.ACT_NONE, out=out)


def linear_swiglu(x, weight, save_pre: bool = False):
    """silu(x @ Wg.T) * (x @ Wu.T) with weight = [Wg; Wu] of shape (2H, D).

    Contract of gko::gemm_swiglu (eval/kernels/gemm_swiglu.py:147-169,
    208-220): x (..., D) -> (..., H), dtype of x. With save_pre, returns (out, gate_up)
    where gate_up = [x Wg^T | x Wu^T] (..., 2H) is written by the same kernel (bf16 / f16).
    """
    dev = _lib.require_cuda(x, weight)
    if weight.dim() != 2 or weight.shape[0] % 2:
        raise RuntimeError(f"gemm_swiglu: weight must be (2H, D), got {tuple(weight.shape)}")
    if x.dtype != weight.dtype:
        raise RuntimeError(f"gemm_swiglu: x {x.dtype} and weight {weight.dtype} differ")
    D = x.shape[-1]
    if weight.shape[1] != D:
        raise RuntimeError(f"gemm_swiglu: shape mismatch x={tuple(x.shape)} weight={tuple(weight.shape)}")
    H = weight.shape[0] // 2
    dt = _lib.dtype_code(x.dtype)
    lead = x.shape[:-1]
    a = x.reshape(-1, D)
    M = a.shape[0]
    if dt != _lib.F32 and a.stride(-1) != 1 and M > 1:
        a = a.contiguous()
    w = weight
    if dt != _lib.F32 and not (w.stride(0) == 1 or w.stride(1) == 1):
        w = w.contiguous()
    out = torch.empty((M, H), device=dev, dtype=x.dtype)
    gu = torch.empty((M, 2 * H), device=dev, dtype=x.dtype) if save_pre else None
    if M and H:
        with torch.cuda.device(dev):
            a_sm = a.stride(0) if M > 1 else max(D, 8)
            if save_pre:
                rc = _lib.load().gko_linear_swiglu_aux(
                    dt, M, H, D, _ptr(a), a_sm, a.stride(1), _ptr(w), w.stride(0), w.stride(1),
                    _ptr(out), out.stride(0), _ptr(gu), gu.stride(0), _status_ptr(dev), _stream(dev),
                )
            else:
                rc = _lib.load().gko_linear_swiglu(
                    dt, M, H, D, _ptr(a), a_sm, a.stride(1), _ptr(w), w.stride(0), w.stride(1),
                    _ptr(out), out.stride(0), _status_ptr(dev), _stream(dev),
                )
        _lib.check(rc, "gko_linear_swiglu_aux" if save_pre else "gko_linear_swiglu")
    if save_pre:
        return out.reshape(*lead, H), gu.reshape(*lead, 2 * H)
    return out.reshape(*lead, H)


def swiglu_bwd(dy, gate_up):
    """[d_gate | d_up] of y = silu(g) * u from dy (..., H) and the saved gate_up = [g | u] (..., 2H)."""
    dev = _lib.require_cuda(dy, gate_up)
    H = dy.shape[-1]
    if gate_up.shape[-1] != 2 * H or gate_up.shape[:-1] != dy.shape[:-1] or dy.dtype != gate_up.dtype:
        raise RuntimeError(f"swiglu_bwd: dy {tuple(dy.shape)} / gate_up {tuple(gate_up.shape)} mismatch")
    d2 = dy.reshape(-1, H).contiguous()
    g2 = gate_up.reshape(-1, 2 * H).contiguous()
    out = torch.empty_like(g2)
    if d2.shape[0] and H:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_swiglu_bwd(
                _lib.dtype_code(dy.dtype), d2.shape[0], H, _ptr(d2), d2.stride(0), _ptr(g2), g2.stride(0),
                _ptr(out), out.stride(0), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_swiglu_bwd")
    return out.reshape(gate_up.shape)


def swiglu_mlp(x, w_gate_up, w_down):
    """(silu(x Wg^T) * (x Wu^T)) Wdown^T: the fused gate/up kernel then the down GEMM."""
    return linear(linear_swiglu(x, w_gate_up), w_down)


def silu_mul(x, y):
    """silu(x) * y elementwise (gko::silu_mul, eval/kernels/silu_mul.py:29-43)."""
    dev = _lib.require_cuda(x, y)
    if x.dtype != y.dtype:
        raise RuntimeError(f"silu_mul: dtypes differ: {x.dtype} vs {y.dtype}")
    if x.shape != y.shape:
        # broadcasting operands (e.g. an SE gate [B, C, 1, 1]) are expanded to the result shape
        shape = torch.broadcast_shapes(x.shape, y.shape)
        x, y = x.expand(shape), y.expand(shape)
    xc = x.contiguous()
    yc = y.contiguous()
    out = torch.empty_like(xc)
    n = xc.numel()
    if n:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_silu_mul(
                _lib.dtype_code(x.dtype), n, _ptr(xc), _ptr(yc), _ptr(out), _status_ptr(dev), _stream(dev)
            )
        _lib.check(rc, "gko_silu_mul")
    return out


def _check_norm_args(name, x, residual=None, weight=None):
    """The norm kernels read rows x cols elements of x, of the residual and cols of the weight, all in x's
    dtype: a residual or weight of another shape or dtype would be read out of bounds or misread."""
    if x.dim() < 1 or x.shape[-1] == 0:
        raise RuntimeError(f"{name}: x needs a non-empty last dim, got {tuple(x.shape)}")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise RuntimeError(f"{name}: residual {tuple(residual.shape)} {residual.dtype} must match x "
                           f"{tuple(x.shape)} {x.dtype}")
    if weight is not None and (weight.numel() != x.shape[-1] or weight.dtype != x.dtype):
        raise RuntimeError(f"{name}: weight {tuple(weight.shape)} {weight.dtype} must have {x.shape[-1]} "
                           f"elements of x's dtype {x.dtype}")


def rmsnorm(x, weight, eps=1e-5, residual=None, return_sum=False):
    """rmsnorm(x (+ residual)) * weight over the last dim; with return_sum also x + residual."""
    dev = _lib.require_cuda(x, weight, residual)
    _check_norm_args("rmsnorm", x, residual, weight)
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols).contiguous()
    r2 = residual.reshape(-1, cols).contiguous() if residual is not None else None
    out = torch.empty(x2.shape, device=dev, dtype=x.dtype)
    total = torch.empty(x2.shape, device=dev, dtype=x.dtype) if (return_sum and r2 is not None) else None
    w = weight.contiguous()
    if x2.shape[0]:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_rmsnorm(
                _lib.dtype_code(x.dtype), x2.shape[0], cols, _ptr(x2), _ptr(r2), _ptr(w), float(eps), _ptr(out),
                _ptr(total), cols, _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_rmsnorm")
    out = out.reshape(x.shape)
    if return_sum:
        return out, (total.reshape(x.shape) if total is not None else x)
    return out


def rope_(x, theta=500000.0, positions=None, seq_len=None):
    """Rotate-half RoPE in place on x [tokens, heads, head_dim] (any token/head strides, unit dim stride).

    Position of token t: positions[t] (int32 tensor) or t % seq_len.
    """
    if x.dim() != 3 or x.stride(-1) != 1:
        raise RuntimeError("rope_: x must be [tokens, heads, head_dim] with unit stride along head_dim")
    t, h, d = x.shape
    if positions is not None and positions.numel() != t:
        raise RuntimeError(f"rope_: positions holds {positions.numel()} entries for {t} tokens")
    dev = _lib.require_cuda(x, positions)
    pos = positions.to(torch.int32).contiguous() if positions is not None else None
    if pos is None and not seq_len:
        seq_len = t
    if t and h:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_rope(
                _lib.dtype_code(x.dtype), t, h, d, _ptr(x), x.stride(0), x.stride(1), _ptr(pos),
                int(seq_len or 0), float(theta), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_rope")
    return x


# --------------------------------------------------------------------------- attention
def _bias_layout(q, k, attn_bias):
    """Map an additive attention bias onto the kernel's bias modes.

    Accepts the layouts of the reference's _bias_pack
    (eval/kernels/fused_sdpa.py:546-575): 1-D/2-D/3-D key padding holding
    z * n_k values, [z|1, 1, 1, n_k] rows, and [z|1|nW, h|1, n_q, n_k] full
    biases with broadcast dims read through stride 0 (no [z, h, n_q, n_k]
    materialisation). Returns (tensor, mode, strides[4], batches).
    """
    z, h, n_q, _ = q.shape
    n_k = k.shape[-2]
    if attn_bias is None or attn_bias.numel() == 0:
        return None, _lib.BIAS_NONE, (0, 0, 0, 0), 1
    b = attn_bias
    if b.dim() <= 2 and b.numel() == z * n_k:
        b = b.reshape(z, n_k)
        return b, _lib.BIAS_KEYPAD, (b.stride(0), 0, 0, b.stride(1)), z
    if b.dim() == 3 and b.shape[-1] == n_k and b.numel() == z * n_k:
        b = b.reshape(z, n_k)
        return b, _lib.BIAS_KEYPAD, (b.stride(0), 0, 0, b.stride(1)), z
    if b.dim() == 4 and b.shape[-2] == 1 and b.shape[-1] == n_k:
        if b.shape[0] == z:
            row = b[:, 0, 0, :]
            return row, _lib.BIAS_KEYPAD, (row.stride(0), 0, 0, row.stride(1)), z
        if b.shape[0] == 1:
            row = b[0, 0, 0, :]
            return row, _lib.BIAS_KEYPAD, (0, 0, 0, row.stride(0)), z
    if b.dim() == 4 and b.shape[-2] == n_q and b.shape[-1] == n_k:
        bz, bh = b.shape[0], b.shape[1]
        if bh not in (1, h):
            raise RuntimeError(f"attention bias head dim {bh} must be 1 or {h}")
        if bz == z:
            nb = z
        elif bz == 1:
            nb = z
        elif z % bz == 0:
            nb = bz  # shifted-window mask [nW, h, n, n] against q [B * nW, h, n, d]
        else:
            raise RuntimeError(f"attention bias batch {bz} does not divide the batch {z}")
        sz = b.stride(0) if bz > 1 else 0
        sh = b.stride(1) if bh > 1 else 0
        sq = b.stride(2) if n_q > 1 else 0
        return b, _lib.BIAS_FULL, (sz, sh, sq, b.stride(3)), nb
    raise RuntimeError(
        f"unsupported attention bias shape {tuple(attn_bias.shape)} for q {tuple(q.shape)}, k {tuple(k.shape)}"
    )


def fmha_fwd(q, k, v, attn_bias=None, scale=None, causal=0, window=0, softcap=0.0, out=None):
    """Fused attention forward -> (out [z, hq, sq, d], lse f32 [z * hq, sq]).

    ``out`` (optional) is a preallocated output with any strides allowed by the kernel (e.g. a
    [z, s, h, d] buffer viewed as [z, h, s, d]); by default a fresh contiguous tensor.

    q [z, hq, sq, d], k/v [z, hkv, sk, d] with hq % hkv == 0 (GQA); any
    strides with unit stride along d (e.g. [z, s, h, d] storage viewed through
    transpose(1, 2)) are read in place. Contract of gko::fused_sdpa_pair
    (eval/kernels/fused_sdpa.py:912-943).
    """
    dev = _lib.require_cuda(q, k, v, attn_bias)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("fmha: q, k, v must be 4-D [z, h, s, d]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise RuntimeError("fmha: q, k, v dtypes differ")
    z, hq, sq, d = q.shape
    _, hkv, sk, dk = k.shape
    if k.shape != v.shape or dk != d or k.shape[0] != z:
        raise RuntimeError(f"fmha: shape mismatch q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if scale is None:
        scale = d ** -0.5
    dt = _lib.dtype_code(q.dtype)

    def _fix(t):
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:3]) or t.data_ptr() % 16:
            return t.contiguous()
        return t

    q, k, v = _fix(q), _fix(k), _fix(v)
    bias_t, mode, bstr, nb = _bias_layout(q, k, attn_bias)
    if out is None:
        out = torch.empty((z, hq, sq, d), device=dev, dtype=q.dtype)
    elif out.shape != (z, hq, sq, d) or out.dtype != q.dtype or out.device != dev:
        raise RuntimeError(f"fmha: out must be [{z}, {hq}, {sq}, {d}] {q.dtype} on {dev}")
    lse = torch.empty((z * hq, sq), device=dev, dtype=torch.float32)
    if z and hq and sq:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_fmha_fwd(
                dt, z, hq, hkv, sq, sk, d,
                _ptr(q), _I64x4(*q.stride()), _ptr(k), _I64x4(*k.stride()), _ptr(v), _I64x4(*v.stride()),
                _ptr(bias_t), mode, _lib.dtype_code(bias_t.dtype) if bias_t is not None else 0,
                _I64x4(*bstr), nb, _I64x4(*out.stride()), float(scale), int(bool(causal)), int(window or 0),
                float(softcap or 0.0),
                _ptr(out), _ptr(lse), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_fmha_fwd")
    return out, lse


def fmha_varlen_fwd(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k=None, scale=None,
                    causal=0, window=0, softcap=0.0):
    """Attention over packed sequences -> (out [tq, hq, d], lse f32 [hq, tq]).

    q [tq, hq, d], k/v [tk, hkv, d]; cu_seqlens_* int32 [b + 1] on the device, non-decreasing from 0 to the
    token count (not checked on the host, which would need a device sync; the kernel writes no row outside
    [0, tq)), and max_seqlen_q at least the longest query sequence.
    """
    dev = _lib.require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise RuntimeError("fmha_varlen: q, k, v must be 3-D [tokens, heads, d]")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise RuntimeError("fmha_varlen: q, k, v dtypes differ")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
        raise RuntimeError("fmha_varlen: cu_seqlens must be int32")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel() or cu_seqlens_q.numel() < 1:
        raise RuntimeError("fmha_varlen: cu_seqlens_q and cu_seqlens_k must both have b + 1 entries")
    tq, hq, d = q.shape
    tk, hkv, dk = k.shape
    if k.shape != v.shape or dk != d:
        raise RuntimeError(f"fmha_varlen: shape mismatch q={tuple(q.shape)} k={tuple(k.shape)}")
    if scale is None:
        scale = d ** -0.5
    b = cu_seqlens_q.numel() - 1

    def _fix(t):
        if t.stride(-1) != 1 or t.stride(0) % 8 or t.stride(1) % 8 or t.data_ptr() % 16:
            return t.contiguous()
        return t

    q, k, v = _fix(q), _fix(k), _fix(v)
    cq = cu_seqlens_q.contiguous()
    ck = cu_seqlens_k.contiguous()
    out = torch.empty((tq, hq, d), device=dev, dtype=q.dtype)
    lse = torch.empty((hq, tq), device=dev, dtype=torch.float32)
    if b and tq and hq:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_fmha_varlen_fwd(
                _lib.dtype_code(q.dtype), b, hq, hkv, d, tq, tk, int(max_seqlen_q),
                _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0),
                v.stride(1), _ptr(cq), _ptr(ck), float(scale), int(bool(causal)), int(window or 0),
                float(softcap or 0.0), _ptr(out), _ptr(lse), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_fmha_varlen_fwd")
    return out, lse


def _bwd_fix(t):
    """Unit d stride, other strides multiples of 8 elements, 16-byte aligned (else a contiguous copy)."""
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
        return t.contiguous()
    return t


def fmha_bwd(q, k, v, attn_bias, out, lse, dout, scale=None, causal=0, window=0, softcap=0.0):
    """Fused attention backward -> (dq, dk, dv), contiguous, dtypes of q / k / v.

    Inputs as for ``fmha_fwd`` plus its ``out`` and ``lse`` and the incoming gradient ``dout``
    [z, hq, sq, d]. Contract of gko::fused_sdpa_bwd (eval/kernels/fused_sdpa.py:945-967); with
    GQA (hkv < hq) dk/dv sum over each kv head's query group. Bias gets no gradient.
    """
    dev = _lib.require_cuda(q, k, v, attn_bias, out, lse, dout)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("fmha_bwd: q, k, v must be 4-D [z, h, s, d]")
    if q.dtype != k.dtype or q.dtype != v.dtype or out.dtype != q.dtype or dout.dtype != q.dtype:
        raise RuntimeError("fmha_bwd: q, k, v, out, dout dtypes differ")
    z, hq, sq, d = q.shape
    _, hkv, sk, dk_ = k.shape
    if k.shape != v.shape or dk_ != d or k.shape[0] != z:
        raise RuntimeError(f"fmha_bwd: shape mismatch q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if out.shape != q.shape or dout.shape != q.shape:
        raise RuntimeError("fmha_bwd: out and dout must have q's shape")
    if lse.dtype != torch.float32 or lse.numel() != z * hq * sq:
        raise RuntimeError("fmha_bwd: lse must be float32 [z * hq, sq]")
    if scale is None:
        scale = d ** -0.5
    dt = _lib.dtype_code(q.dtype)
    q, k, v, out, dout = (_bwd_fix(t) for t in (q, k, v, out, dout))
    lse = lse.contiguous()
    bias_t, mode, bstr, nb = _bias_layout(q, k, attn_bias)
    dq = torch.empty((z, hq, sq, d), device=dev, dtype=q.dtype)
    dk = torch.empty((z, hkv, sk, d), device=dev, dtype=k.dtype)
    dv = torch.empty((z, hkv, sk, d), device=dev, dtype=v.dtype)
    if z and hq and (sq or sk):
        lib = _lib.load()
        ws_bytes = lib.gko_fmha_bwd_workspace_size(z, hq, sq, d, 0)
        if ws_bytes < 0:
            _lib.check(_lib.ERR_UNSUPPORTED, "gko_fmha_bwd_workspace_size")
        ws = torch.empty(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            rc = lib.gko_fmha_bwd(
                dt, z, hq, hkv, sq, sk, d,
                _ptr(q), _I64x4(*q.stride()), _ptr(k), _I64x4(*k.stride()), _ptr(v), _I64x4(*v.stride()),
                _ptr(bias_t), mode, _lib.dtype_code(bias_t.dtype) if bias_t is not None else 0,
                _I64x4(*bstr), nb, _ptr(out), _I64x4(*out.stride()), _ptr(dout), _I64x4(*dout.stride()),
                _ptr(lse), float(scale), int(bool(causal)), int(window or 0), float(softcap or 0.0),
                _ptr(dq), _I64x4(*dq.stride()), _ptr(dk), _I64x4(*dk.stride()), _ptr(dv), _I64x4(*dv.stride()),
                _ptr(ws), ws_bytes, _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_fmha_bwd")
    return dq, dk, dv


def fmha_varlen_bwd(q, k, v, out, lse, dout, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, scale=None,
                    causal=0, window=0, softcap=0.0):
    """Backward of ``fmha_varlen_fwd`` -> (dq [tq, hq, d], dk, dv [tk, hkv, d]). cu_seqlens must be
    non-decreasing from 0 to the token counts, as for the forward; the kernels clamp every
    sequence's rows to [0, tq) / [0, tk), so malformed cu_seqlens give wrong gradients but no
    access outside the tensors and the workspace."""
    dev = _lib.require_cuda(q, k, v, out, lse, dout, cu_seqlens_q, cu_seqlens_k)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise RuntimeError("fmha_varlen_bwd: q, k, v must be 3-D [tokens, heads, d]")
    if q.dtype != k.dtype or q.dtype != v.dtype or out.dtype != q.dtype or dout.dtype != q.dtype:
        raise RuntimeError("fmha_varlen_bwd: q, k, v, out, dout dtypes differ")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
        raise RuntimeError("fmha_varlen_bwd: cu_seqlens must be int32")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel() or cu_seqlens_q.numel() < 1:
        raise RuntimeError("fmha_varlen_bwd: cu_seqlens_q and cu_seqlens_k must both have b + 1 entries")
    tq, hq, d = q.shape
    tk, hkv, dk_ = k.shape
    if k.shape != v.shape or dk_ != d or out.shape != q.shape or dout.shape != q.shape:
        raise RuntimeError(f"fmha_varlen_bwd: shape mismatch q={tuple(q.shape)} k={tuple(k.shape)}")
    if lse.dtype != torch.float32 or lse.numel() != hq * tq:
        raise RuntimeError("fmha_varlen_bwd: lse must be float32 [hq, tq]")
    if scale is None:
        scale = d ** -0.5
    b = cu_seqlens_q.numel() - 1
    q, k, v, out, dout = (_bwd_fix(t) for t in (q, k, v, out, dout))
    lse = lse.contiguous()
    cq = cu_seqlens_q.contiguous()
    ck = cu_seqlens_k.contiguous()
    dq = torch.empty((tq, hq, d), device=dev, dtype=q.dtype)
    dk = torch.empty((tk, hkv, d), device=dev, dtype=k.dtype)
    dv = torch.empty((tk, hkv, d), device=dev, dtype=v.dtype)
    if b and hq and (tq or tk):
        lib = _lib.load()
        ws_bytes = lib.gko_fmha_bwd_workspace_size(b, hq, tq, d, 1)
        if ws_bytes < 0:
            _lib.check(_lib.ERR_UNSUPPORTED, "gko_fmha_bwd_workspace_size")
        ws = torch.empty(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            rc = lib.gko_fmha_varlen_bwd(
                _lib.dtype_code(q.dtype), b, hq, hkv, d, tq, tk, int(max_seqlen_q), int(max_seqlen_k),
                _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0),
                v.stride(1), _ptr(out), out.stride(0), out.stride(1), _ptr(dout), dout.stride(0), dout.stride(1),
                _ptr(lse), _ptr(cq), _ptr(ck), float(scale), int(bool(causal)), int(window or 0),
                float(softcap or 0.0), _ptr(dq), dq.stride(0), dq.stride(1), _ptr(dk), dk.stride(0), dk.stride(1),
                _ptr(dv), dv.stride(0), dv.stride(1), _ptr(ws), ws_bytes, _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_fmha_varlen_bwd")
    return dq, dk, dv


# --------------------------------------------------------------------------- tensor-parallel GEMM + all-reduce
def linear_allreduce(x, weight, out, multicast_ptr: int, peers_dev_ptr: int, world: int):
    """out of every rank += x @ weight^T, inside the GEMM (see evocompile_b200.tp).

    ``out`` is this rank's copy of a symmetric-memory buffer, already zeroed on every rank;
    ``multicast_ptr`` its NVLink multicast address (0 if none) and ``peers_dev_ptr`` the device
    array of all ranks' copies. The caller orders the zeroing and the completion with group
    barriers.
    """
    dev = _lib.require_cuda(x, weight, out)
    if x.dim() != 2 or weight.dim() != 2 or out.dim() != 2:
        raise RuntimeError("linear_allreduce: x [m, k], weight [n, k], out [m, n]")
    if x.dtype != weight.dtype or x.dtype != out.dtype:
        raise RuntimeError("linear_allreduce: x, weight, out dtypes differ")
    m, k = x.shape
    n = weight.shape[0]
    if weight.shape[1] != k or tuple(out.shape) != (m, n):
        raise RuntimeError(f"linear_allreduce: shape mismatch x {tuple(x.shape)} weight {tuple(weight.shape)} "
                           f"out {tuple(out.shape)}")
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    if m and n:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_linear_allreduce(
                _lib.dtype_code(x.dtype), m, n, k, _ptr(x), x.stride(0), 1, _ptr(weight), weight.stride(0), 1,
                _ptr(out), out.stride(0), ctypes.c_void_p(multicast_ptr or 0), ctypes.c_void_p(peers_dev_ptr or 0),
                int(world), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_linear_allreduce")
    return out


def linear_residual(x, weight, resid, out=None):
    """x @ weight^T + resid with the residual add in the GEMM epilogue (gko_linear_residual).

    x [m, k] and weight [n, k] row-major, resid [m, n]; bf16 / f16. ``out`` (default: a new
    tensor) may be ``resid`` itself for an in-place residual update, but must not overlap
    x or weight. Returns out.
    """
    if out is not None:
        _check_no_overlap("linear_residual", out, x=x, weight=weight)
    dev = _lib.require_cuda(x, weight, resid, out)
    if x.dim() != 2 or weight.dim() != 2 or resid.dim() != 2:
        raise RuntimeError("linear_residual: x [m, k], weight [n, k], resid [m, n]")
    if x.dtype != weight.dtype or x.dtype != resid.dtype:
        raise RuntimeError("linear_residual: x, weight, resid dtypes differ")
    m, k = x.shape
    n = weight.shape[0]
    if weight.shape[1] != k or tuple(resid.shape) != (m, n):
        raise RuntimeError(f"linear_residual: shape mismatch x {tuple(x.shape)} weight {tuple(weight.shape)} "
                           f"resid {tuple(resid.shape)}")
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=x.dtype)
    elif tuple(out.shape) != (m, n) or out.dtype != x.dtype or out.stride(1) != 1:
        raise RuntimeError("linear_residual: out must be a row-major [m, n] tensor of x's dtype")
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    if resid.stride(1) != 1:
        resid = resid.contiguous()
    if m and n:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_linear_residual(
                _lib.dtype_code(x.dtype), m, n, k, _ptr(x), x.stride(0), 1, _ptr(weight), weight.stride(0), 1,
                _ptr(resid), resid.stride(0), _ptr(out), out.stride(0), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_linear_residual")
    return out


def rms_stats(x, eps=1e-5, residual=None):
    """Per-row 1 / sqrt(mean(v^2) + eps) of v = x (+ residual), fp32 [rows]; with a residual also
    returns v (the updated residual stream) as (inv, v). x [..., cols] bf16 / f16."""
    dev = _lib.require_cuda(x, residual)
    _check_norm_args("rms_stats", x, residual)
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols).contiguous()
    r2 = residual.reshape(-1, cols).contiguous() if residual is not None else None
    inv = torch.empty(x2.shape[0], device=dev, dtype=torch.float32)
    total = torch.empty(x2.shape, device=dev, dtype=x.dtype) if r2 is not None else None
    if x2.shape[0]:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_rms_stats(
                _lib.dtype_code(x.dtype), x2.shape[0], cols, _ptr(x2), _ptr(r2), float(eps), _ptr(total), _ptr(inv),
                cols, _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_rms_stats")
    if r2 is not None:
        return inv, total.reshape(x.shape)
    return inv


def fold_rmsnorm_weight(weight, norm_weight):
    """w'[n, j] = w[n, j] * g[j] (computed in fp32, rounded once): the projection weight that,
    with rms_stats' per-row scale in linear_rowscale, applies RMSNorm(g) before the projection."""
    return (weight.float() * norm_weight.float().view(1, -1)).to(weight.dtype)


def linear_rowscale(x, weight, row_scale, swiglu: bool = False, rope=None):
    """out = row_scale[:, None] * (x @ weight^T) on the tensor-core GEMM (the scale applied to the
    accumulator in the epilogue); with swiglu, weight = [Wg; Wu] (2H, K) and
    out = silu(s x Wg^T) * (s x Wu^T) (rows, H). x [rows, K] row-major, row_scale fp32 [rows].

    ``rope = (rope_cols, seq_len, theta)`` also rotates output columns [0, rope_cols) (heads of
    128) with rotate-half RoPE at position row % seq_len, in the epilogue (gko_linear_rowscale_rope)."""
    dev = _lib.require_cuda(x, weight, row_scale)
    if x.dim() != 2 or weight.dim() != 2 or row_scale.dim() != 1:
        raise RuntimeError("linear_rowscale: x [m, k], weight [n, k], row_scale [m]")
    if x.dtype != weight.dtype or row_scale.dtype != torch.float32:
        raise RuntimeError("linear_rowscale: x and weight share a dtype; row_scale is float32")
    m, k = x.shape
    if weight.shape[1] != k or row_scale.shape[0] != m:
        raise RuntimeError(f"linear_rowscale: shape mismatch x {tuple(x.shape)} weight {tuple(weight.shape)} "
                           f"row_scale {tuple(row_scale.shape)}")
    if swiglu and weight.shape[0] % 2:
        raise RuntimeError("linear_rowscale: the SwiGLU weight has an even number of rows [Wg; Wu]")
    n = weight.shape[0] // 2 if swiglu else weight.shape[0]
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    row_scale = row_scale.contiguous()
    out = torch.empty(m, n, device=x.device, dtype=x.dtype)
    if rope is not None:
        if swiglu:
            raise RuntimeError("linear_rowscale: RoPE applies to the plain (non-SwiGLU) projection only")
        rope_cols, seq_len, theta = rope
        if m and n:
            with torch.cuda.device(dev):
                rc = _lib.load().gko_linear_rowscale_rope(
                    _lib.dtype_code(x.dtype), m, n, k, _ptr(x), x.stride(0), 1, _ptr(weight), weight.stride(0), 1,
                    _ptr(row_scale), _ptr(out), out.stride(0), int(rope_cols), int(seq_len), float(theta),
                    _status_ptr(dev), _stream(dev),
                )
            _lib.check(rc, "gko_linear_rowscale_rope")
        return out
    if m and n:
        with torch.cuda.device(dev):
            rc = _lib.load().gko_linear_rowscale(
                _lib.dtype_code(x.dtype), int(bool(swiglu)), m, n, k, _ptr(x), x.stride(0), 1, _ptr(weight),
                weight.stride(0), 1, _ptr(row_scale), _ptr(out), out.stride(0), _status_ptr(dev), _stream(dev),
            )
        _lib.check(rc, "gko_linear_rowscale")
    return out
