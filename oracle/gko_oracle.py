"""CPU oracle for the fused operators — TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch fp32 on the CPU, the reference's eager
formulas for the three fused operators (file:line into the EvoCompile
repository given per function). Only tests, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it, and only as the checker or the
timed CPU baseline; the product path (``evocompile_b200``) never calls it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Python ops
(imported from the reference checkout on the CPU) on seeded inputs and stores
the outputs as fixtures; ``tests/test_oracle_golden.py`` checks this module
against them. GQA, varlen and the window/softcap semantics of the Triton
kernel have no reference CPU path that covers them all; where a fixture could
not come from the reference the test says so.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = [
    "addmm_gelu",
    "addmm_act",
    "gemm_swiglu",
    "swiglu_mlp",
    "silu_mul",
    "attention",
    "attention_varlen",
    "attention_bwd",
    "attention_varlen_bwd",
    "rmsnorm",
    "rope",
    "llama_block",
]


def _f32(t):
    # no detach: the backward restatements differentiate through these functions
    return None if t is None else t.to("cpu", torch.float32)


def addmm_act(bias, mat1, mat2, act: str = "gelu"):
    """act(mat1 @ mat2 + bias) in fp32.

    Restates _eager_addmm_gelu (eval/kernels/addmm_gelu.py:81-84):
    ``gelu(addmm(bias, m1, m2), approximate='none')`` for 2-D operands and
    ``gelu(matmul(m1, m2) + bias)`` otherwise. ``act`` in {"gelu", "relu", "none"}.
    """
    b, a, w = _f32(bias), _f32(mat1), _f32(mat2)
    if a.dim() == 2 and b is not None:
        z = torch.addmm(b, a, w)
    else:
        z = torch.matmul(a, w)
        if b is not None:
            z = z + b
    if act == "gelu":
        return F.gelu(z, approximate="none")
    if act == "relu":
        return torch.relu(z)
    return z


def addmm_gelu(bias, mat1, mat2):
    return addmm_act(bias, mat1, mat2, "gelu")


def gemm_swiglu(x, weight):
    """silu(x Wg^T) * (x Wu^T), weight = [Wg; Wu] (2H, D), in fp32.

    Restates _eager_gemm_swiglu (eval/kernels/gemm_swiglu.py:105-109).
    """
    gate_up = F.linear(_f32(x), _f32(weight))
    gate, up = gate_up.chunk(2, dim=-1)
    return F.silu(gate) * up


def swiglu_mlp(x, w_gate_up, w_down):
    """SwiGLU MLP: gemm_swiglu followed by the down projection ``F.linear(h, Wdown)``
    (the caller-side c_proj of eval/rewrites/simple_gpt_silu_mul.py:11-18)."""
    return F.linear(gemm_swiglu(x, w_gate_up), _f32(w_down))


def silu_mul(x, y):
    """silu(x) * y (eval/kernels/silu_mul.py:29-30)."""
    return F.silu(_f32(x)) * _f32(y)


def _expand_bias(bias, z, h, n_q, n_k):
    """Bias layouts accepted by the reference's _bias_pack (eval/kernels/fused_sdpa.py:546-575),
    returned as a dense [z, h, n_q, n_k] fp32 tensor."""
    if bias is None or bias.numel() == 0:
        return None
    b = _f32(bias)
    if b.dim() <= 2 and b.numel() == z * n_k:
        return b.reshape(z, 1, 1, n_k).expand(z, h, n_q, n_k)
    if b.dim() == 3 and b.shape[-1] == n_k and b.numel() == z * n_k:
        return b.reshape(z, 1, 1, n_k).expand(z, h, n_q, n_k)
    if b.dim() == 4 and b.shape[-2] == 1 and b.shape[-1] == n_k:
        row = b[:, 0, 0, :] if b.shape[0] == z else b[0, 0, 0, :].expand(z, n_k)
        return row.reshape(z, 1, 1, n_k).expand(z, h, n_q, n_k)
    if b.dim() == 4 and b.shape[-2] == n_q and b.shape[-1] == n_k:
        if b.shape[0] == 1:
            b = b.expand(z, b.shape[1], n_q, n_k)
        elif b.shape[0] != z:
            b = b.repeat(z // b.shape[0], 1, 1, 1)
        return b.expand(z, h, n_q, n_k)
    raise ValueError(f"unsupported bias shape {tuple(bias.shape)}")


def attention(q, k, v, attn_bias=None, scale=None, causal=0, window=0, softcap=0.0):
    """Attention forward in fp32 -> (out [z, hq, sq, d], lse [z * hq, sq]).

    Restates the reference Triton kernel _flash_fwd (eval/kernels/fused_sdpa.py:
    107-157) as one dense computation: logits = scale * q k^T (:108), + bias
    (:109-123), softcap = softcap * tanh(clamp(x / softcap, -15, 15)) (:124-128),
    masks for keys beyond n_k, causal key <= query (:130-135, top-left aligned)
    and |key - query| <= window (:136-138); softmax; lse = max + ln(sum) (:157).
    GQA (k/v with fewer heads) repeats each kv head over its query group —
    an addition, the reference requires equal heads (:535-543). Masked logits are
    removed (not set to -1e6): a row with every key masked gives zeros and
    lse = -inf, where the reference Triton would average the masked keys.
    """
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    z, hq, n_q, d = qf.shape
    hkv, n_k = kf.shape[1], kf.shape[2]
    if scale is None:
        scale = d ** -0.5
    if hkv != hq:
        g = hq // hkv
        kf = kf.repeat_interleave(g, dim=1)
        vf = vf.repeat_interleave(g, dim=1)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * float(scale)
    b = _expand_bias(attn_bias, z, hq, n_q, n_k)
    if b is not None:
        s = s + b
    if softcap and float(softcap) > 0:
        sc = float(softcap)
        s = sc * torch.tanh(torch.clamp(s / sc, -15.0, 15.0))
    qi = torch.arange(n_q)[:, None]
    ki = torch.arange(n_k)[None, :]
    keep = torch.ones(n_q, n_k, dtype=torch.bool)
    if causal:
        keep &= ki <= qi
    if window and int(window) > 0:
        w = int(window)
        keep &= (ki - qi <= w) & (qi - ki <= w)
    s = s.masked_fill(~keep, float("-inf"))
    m = s.amax(dim=-1, keepdim=True)
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp(s - m_safe)
    l = p.sum(dim=-1, keepdim=True)
    out = torch.matmul(p, vf) / torch.where(l > 0, l, torch.ones_like(l))
    out = torch.where(l > 0, out, torch.zeros_like(out))
    lse = torch.where(l > 0, m_safe + torch.log(l), torch.full_like(l, float("-inf")))
    return out, lse.reshape(z * hq, n_q)


def attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, scale=None, causal=0, window=0, softcap=0.0):
    """Packed variable-length attention in fp32 -> (out [tq, hq, d], lse [hq, tq]).

    One dense ``attention`` call per sequence (no reference counterpart: the
    reference attention takes only dense batches).
    """
    qf, kf, vf = _f32(q), _f32(k), _f32(v)
    tq, hq, d = qf.shape
    cq = [int(x) for x in cu_seqlens_q.tolist()]
    ck = [int(x) for x in cu_seqlens_k.tolist()]
    out = torch.zeros(tq, hq, d)
    lse = torch.full((hq, tq), float("-inf"))
    for i in range(len(cq) - 1):
        q0, q1, k0, k1 = cq[i], cq[i + 1], ck[i], ck[i + 1]
        if q1 <= q0:
            continue
        qs = qf[q0:q1].transpose(0, 1).unsqueeze(0)
        ks = kf[k0:k1].transpose(0, 1).unsqueeze(0)
        vs = vf[k0:k1].transpose(0, 1).unsqueeze(0)
        o, l = attention(qs, ks, vs, None, scale, causal, window, softcap)
        out[q0:q1] = o[0].transpose(0, 1)
        lse[:, q0:q1] = l.reshape(hq, q1 - q0)
    return out, lse


def attention_bwd(q, k, v, dout, attn_bias=None, scale=None, causal=0, window=0, softcap=0.0):
    """(dq, dk, dv) in fp32 for upstream gradient ``dout`` of ``attention``'s output.

    Autograd of the fp32 restatement above, i.e. the math the reference's backward
    kernels compute (eval/kernels/fused_sdpa.py:159-496 with the launch sequence of
    _triton_bwd at :668-770): delta = rowsum(O dO), P = exp(logits - lse),
    dv = P^T dO, dS = P (dP - delta) (times the softcap derivative), dq = scale dS k,
    dk = scale dS^T q. GQA gradients sum over each kv head's query group. The bias
    gets no gradient (the reference returns None for it, :865-870).
    """
    qf, kf, vf = (_f32(t).clone().requires_grad_(True) for t in (q, k, v))
    with torch.enable_grad():
        out, _ = attention(qf, kf, vf, attn_bias, scale, causal, window, softcap)
        out.backward(_f32(dout))
    return qf.grad, kf.grad, vf.grad


def attention_varlen_bwd(q, k, v, dout, cu_seqlens_q, cu_seqlens_k, scale=None, causal=0, window=0, softcap=0.0):
    """(dq, dk, dv) in fp32 of ``attention_varlen`` for upstream gradient ``dout`` (autograd)."""
    qf, kf, vf = (_f32(t).clone().requires_grad_(True) for t in (q, k, v))
    with torch.enable_grad():
        out, _ = attention_varlen(qf, kf, vf, cu_seqlens_q, cu_seqlens_k, scale, causal, window, softcap)
        out.backward(_f32(dout))
    return qf.grad, kf.grad, vf.grad


def rel_err(out, ref) -> float:
    """max |out - ref| / max |ref| (the bf16 tolerance metric)."""
    o = _f32(out)
    r = _f32(ref)
    denom = r.abs().max().item()
    if denom == 0:
        return o.abs().max().item()
    return (o - r).abs().max().item() / denom


def scaled_tolerance_ok(out, ref, rel: float) -> bool:
    return rel_err(out, ref) <= rel and not math.isnan(rel_err(out, ref))


def rmsnorm(x, weight, eps=1e-5):
    """x * rsqrt(mean(x^2) + eps) * weight over the last dim, fp32 (Llama RMSNorm)."""
    xf = _f32(x)
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * _f32(weight)


def rope(x, theta=500000.0, positions=None):
    """Rotate-half RoPE (the HF Llama convention) of x [tokens, heads, D] in fp32 at positions[t]."""
    xf = _f32(x)
    t, _, d = xf.shape
    pos = torch.arange(t, dtype=torch.float64) if positions is None else _f32(positions).double()
    inv_freq = torch.pow(torch.tensor(theta, dtype=torch.float64), -torch.arange(0, d, 2, dtype=torch.float64) / d)
    ang = (pos[:, None] * inv_freq[None, :]).float()          # [t, D/2]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def llama_block(x, w, cfg):
    """One Llama transformer block (prefill, causal, GQA) in fp32 on the CPU.

    x [B, S, d]; w holds the full weights (attn_norm, wq, wk, wv, wo, mlp_norm, w_gate, w_up, w_down);
    cfg has d_model, n_heads, n_kv_heads, head_dim, d_ff, eps, rope_theta. No reference counterpart
    (the reference's kernel path has no block); this is the standard formulation the fused path computes.
    """
    xf = _f32(x)
    B, S, d = xf.shape
    hd = cfg.head_dim
    h = rmsnorm(xf, w["attn_norm"], cfg.eps)
    q = F.linear(h, _f32(w["wq"])).view(B, S, cfg.n_heads, hd)
    k = F.linear(h, _f32(w["wk"])).view(B, S, cfg.n_kv_heads, hd)
    v = F.linear(h, _f32(w["wv"])).view(B, S, cfg.n_kv_heads, hd)
    pos = torch.arange(S)
    q = torch.stack([rope(q[b], cfg.rope_theta, pos) for b in range(B)])
    k = torch.stack([rope(k[b], cfg.rope_theta, pos) for b in range(B)])
    # attention one kv group at a time (its query heads against its one kv head): the same math,
    # with the [B, heads, S, S] logits held for one group only
    g = cfg.n_heads // cfg.n_kv_heads
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    o = torch.cat([attention(qh[:, j * g:(j + 1) * g], kh[:, j:j + 1], vh[:, j:j + 1], None, hd ** -0.5, 1)[0]
                   for j in range(cfg.n_kv_heads)], dim=1)
    o = F.linear(o.transpose(1, 2).reshape(B, S, cfg.n_heads * hd), _f32(w["wo"]))
    x1 = xf + o
    h2 = rmsnorm(x1, w["mlp_norm"], cfg.eps)
    g = F.silu(F.linear(h2, _f32(w["w_gate"]))) * F.linear(h2, _f32(w["w_up"]))
    return x1 + F.linear(g, _f32(w["w_down"]))
