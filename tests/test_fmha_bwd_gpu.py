"""Parity of the tcgen05 attention backward (gko_fmha_bwd / gko_fmha_varlen_bwd) against
the fp32 oracle (autograd of the CPU restatement), through the C ABI.

The forward output and lse that the backward consumes come from the library's own
forward, as in training. bf16/fp16 gradients: max|err| / max|ref| <= 3e-2 for each of
dq, dk, dv (P and dS enter the tensor core as bf16/fp16, one rounding more than the
forward's output).
"""

import pytest
import torch

import oracle
from evocompile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 3e-2


def _inputs(seed, z, hq, hkv, sq, sk, d, dtype, layout="bhsd"):
    g = torch.Generator().manual_seed(seed)
    if layout == "bhsd":
        mk = lambda h, s: torch.randn(z, h, s, d, generator=g).to(dtype)  # noqa: E731
        to_dev = lambda t: t.cuda()  # noqa: E731
    else:  # [z, s, h, d] storage viewed as [z, h, s, d]
        mk = lambda h, s: torch.randn(z, s, h, d, generator=g).to(dtype).transpose(1, 2)  # noqa: E731
        to_dev = lambda t: t.transpose(1, 2).contiguous().cuda().transpose(1, 2)  # noqa: E731
    q, k, v = mk(hq, sq), mk(hkv, sk), mk(hkv, sk)
    dout = mk(hq, sq)
    return q, k, v, dout, to_dev


def _run(q, k, v, dout, to_dev, bias=None, scale=None, causal=0, window=0, softcap=0.0):
    qd, kd, vd, dod = to_dev(q), to_dev(k), to_dev(v), to_dev(dout)
    bd = bias.cuda() if bias is not None else None
    out, lse = ops.fmha_fwd(qd, kd, vd, bd, scale, causal, window, softcap)
    dq, dk, dv = ops.fmha_bwd(qd, kd, vd, bd, out, lse, dod, scale, causal, window, softcap)
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0, "a kernel reported a timeout"
    return dq, dk, dv


def _check(got, ref):
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        assert g.shape == r.shape, name
        assert torch.isfinite(g.float()).all(), name
        err = oracle.rel_err(g, r)
        assert err <= TOL, f"{name}: rel err {err:.4f}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("s", [1, 64, 200, 333])
def test_bwd_dense(dtype, d, causal, s):
    q, k, v, do, dev = _inputs(s * 10 + d + causal, 2, 2, 2, s, s, d, dtype)
    ref = oracle.attention_bwd(q, k, v, do, None, d ** -0.5, causal)
    _check(_run(q, k, v, do, dev, None, d ** -0.5, causal), ref)


@pytest.mark.parametrize("sq,sk", [(64, 300), (300, 64), (100, 400), (129, 1000)])
@pytest.mark.parametrize("causal", [0, 1])
def test_bwd_cross_lengths(sq, sk, causal):
    """Includes causal sq < sk, where keys past the last query get zero dk / dv."""
    q, k, v, do, dev = _inputs(sq + sk + causal, 1, 2, 2, sq, sk, 128, torch.bfloat16)
    ref = oracle.attention_bwd(q, k, v, do, None, 0.1, causal)
    _check(_run(q, k, v, do, dev, None, 0.1, causal), ref)


@pytest.mark.parametrize("hq,hkv", [(8, 2), (8, 1), (4, 4)])
def test_bwd_gqa_bshd_layout(hq, hkv):
    q, k, v, do, dev = _inputs(hq * 7 + hkv, 2, hq, hkv, 300, 300, 128, torch.bfloat16, layout="bshd")
    ref = oracle.attention_bwd(q, k, v, do, None, 128 ** -0.5, 1)
    _check(_run(q, k, v, do, dev, None, 128 ** -0.5, 1), ref)


@pytest.mark.parametrize("kind", ["keypad", "keypad4d", "full", "full_bcast", "swin"])
def test_bwd_bias(kind):
    z, h, s, d = 4, 2, 150, 64
    q, k, v, do, dev = _inputs(37, z, h, h, s, s, d, torch.bfloat16)
    g = torch.Generator().manual_seed(6)
    if kind == "keypad":
        bias = torch.zeros(z, s)
        bias[:, -20:] = float("-inf")
        bias = bias.to(torch.bfloat16)
    elif kind == "keypad4d":
        bias = torch.randn(z, 1, 1, s, generator=g).to(torch.bfloat16)
    elif kind == "full":
        bias = torch.randn(z, h, s, s, generator=g)
    elif kind == "full_bcast":
        bias = torch.randn(1, 1, s, s, generator=g).to(torch.bfloat16)
    else:
        bias = torch.randn(2, h, s, s, generator=g).to(torch.bfloat16)
    ref = oracle.attention_bwd(q, k, v, do, bias, 0.125, 0)
    _check(_run(q, k, v, do, dev, bias, 0.125, 0), ref)


@pytest.mark.parametrize("window,causal,softcap", [(32, 0, 0.0), (100, 1, 0.0), (0, 1, 30.0), (50, 0, 5.0)])
def test_bwd_window_softcap(window, causal, softcap):
    q, k, v, do, dev = _inputs(window + causal + 3, 2, 2, 2, 400, 400, 128, torch.bfloat16)
    ref = oracle.attention_bwd(q, k, v, do, None, 128 ** -0.5, causal, window, softcap)
    _check(_run(q, k, v, do, dev, None, 128 ** -0.5, causal, window, softcap), ref)


def test_bwd_fully_masked_rows():
    """Batch 0 has every key masked: its gradients are exactly zero."""
    z, h, s, d = 2, 2, 70, 64
    q, k, v, do, dev = _inputs(4, z, h, h, s, s, d, torch.bfloat16)
    bias = torch.zeros(z, s)
    bias[0, :] = float("-inf")
    ref = oracle.attention_bwd(q, k, v, do, bias, 0.125, 0)
    got = _run(q, k, v, do, dev, bias, 0.125, 0)
    _check(got, ref)
    for g in got:
        assert g[0].abs().max().item() == 0.0


@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("hq,hkv", [(8, 2), (4, 4)])
def test_bwd_varlen(causal, hq, hkv):
    lens = [1, 65, 0, 300, 128, 7, 513]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    t = int(cu[-1])
    g = torch.Generator().manual_seed(len(lens) + hq + causal)
    q = torch.randn(t, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(t, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(t, hkv, 128, generator=g).to(torch.bfloat16)
    do = torch.randn(t, hq, 128, generator=g).to(torch.bfloat16)
    ref = oracle.attention_varlen_bwd(q, k, v, do, cu, cu, 128 ** -0.5, causal)
    cud = cu.cuda()
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    out, lse = ops.fmha_varlen_fwd(qd, kd, vd, cud, cud, max(lens), max(lens), 128 ** -0.5, causal)
    got = ops.fmha_varlen_bwd(qd, kd, vd, out, lse, dod, cud, cud, max(lens), max(lens), 128 ** -0.5, causal)
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0
    _check(got, ref)


def test_bwd_dropin_autograd():
    """fused_attention(...).backward() runs the library backward through gko::fused_sdpa_bwd."""
    from evocompile_b200.kernels import fused_sdpa

    q, k, v, do, dev = _inputs(11, 2, 4, 4, 256, 256, 128, torch.bfloat16, layout="bshd")
    ref = oracle.attention_bwd(q, k, v, do, None, 128 ** -0.5, 1)
    qd, kd, vd = (dev(t).detach().requires_grad_(True) for t in (q, k, v))
    out = fused_sdpa.fused_attention(qd, kd, vd, None, 128 ** -0.5, 1)
    out.backward(dev(do))
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0
    _check((qd.grad, kd.grad, vd.grad), ref)


def test_bwd_repeatable_and_workspace_reuse():
    """Two calls (fresh workspace each) agree to fp32 summation-order noise."""
    q, k, v, do, dev = _inputs(5, 2, 4, 2, 513, 513, 128, torch.bfloat16)
    a = _run(q, k, v, do, dev, None, None, 1)
    b = _run(q, k, v, do, dev, None, None, 1)
    for x, y in zip(a, b):
        assert oracle.rel_err(x, y) <= 1e-2


@pytest.mark.slow
def test_bwd_full_config_sampled_heads():
    """Causal backward at B=8, H=32, S=4096, D=128 in [B,S,H,D] layout; an fp32 torch
    reference on the GPU checks three (batch, head) slices."""
    torch.manual_seed(1)
    dev = torch.device("cuda", 0)
    B, S, H, D = 8, 4096, 32, 128
    mk = lambda: torch.randn(B, S, H, D, device=dev).to(torch.bfloat16).transpose(1, 2)  # noqa: E731
    q, k, v, do = mk(), mk(), mk(), mk()
    out, lse = ops.fmha_fwd(q, k, v, None, D ** -0.5, 1)
    dq, dk, dv = ops.fmha_bwd(q, k, v, None, out, lse, do, D ** -0.5, 1)
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    mask = torch.ones(S, S, dtype=torch.bool, device=dev).tril()
    for b, h in [(0, 0), (3, 17), (7, 31)]:
        qs, ks, vs = (t[b, h].float().requires_grad_(True) for t in (q, k, v))
        s = (qs @ ks.T) * D ** -0.5
        p = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=-1)
        (p @ vs).backward(do[b, h].float())
        for g, r in ((dq[b, h], qs.grad), (dk[b, h], ks.grad), (dv[b, h], vs.grad)):
            assert oracle.rel_err(g, r) <= TOL


@pytest.mark.parametrize("causal", [0, 1])
def test_bwd_varlen_edges_write_nothing_outside(causal):
    """Valid edge cases of cu_seqlens (empty and one-token sequences, the last sequence ending
    exactly at the packed token count): dq, dk, dv and the workspace are the heads of larger
    buffers whose tails hold a canary; the kernels write only inside the tensors."""
    import ctypes

    lens = [0, 1, 1, 64, 0, 130, 1, 200]
    hq, hkv, d = 4, 2, 128
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    t = int(cu[-1])
    g = torch.Generator().manual_seed(71 + causal)
    q = torch.randn(t, hq, d, generator=g).to(torch.bfloat16)
    k = torch.randn(t, hkv, d, generator=g).to(torch.bfloat16)
    v = torch.randn(t, hkv, d, generator=g).to(torch.bfloat16)
    do = torch.randn(t, hq, d, generator=g).to(torch.bfloat16)
    ref = oracle.attention_varlen_bwd(q, k, v, do, cu, cu, d ** -0.5, causal)
    cud = cu.cuda()
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    out, lse = ops.fmha_varlen_fwd(qd, kd, vd, cud, cud, max(lens), max(lens), d ** -0.5, causal)
    canary = 7.0
    tail = 4096
    bq = torch.full((t * hq * d + tail,), canary, dtype=torch.bfloat16, device="cuda")
    bk = torch.full((t * hkv * d + tail,), canary, dtype=torch.bfloat16, device="cuda")
    bv = torch.full((t * hkv * d + tail,), canary, dtype=torch.bfloat16, device="cuda")
    dq, dk, dv = bq[: t * hq * d].view(t, hq, d), bk[: t * hkv * d].view(t, hkv, d), bv[: t * hkv * d].view(t, hkv, d)
    lib = _lib.load()
    ws_bytes = lib.gko_fmha_bwd_workspace_size(len(lens), hq, t, d, 1)
    wsb = torch.full((ws_bytes // 4 + tail,), canary, dtype=torch.float32, device="cuda")
    vp = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    dev = torch.device("cuda", 0)
    rc = lib.gko_fmha_varlen_bwd(
        _lib.dtype_code(q.dtype), len(lens), hq, hkv, d, t, t, max(lens), max(lens),
        vp(qd), qd.stride(0), qd.stride(1), vp(kd), kd.stride(0), kd.stride(1), vp(vd), vd.stride(0), vd.stride(1),
        vp(out), out.stride(0), out.stride(1), vp(dod), dod.stride(0), dod.stride(1), vp(lse), vp(cud), vp(cud),
        float(d ** -0.5), causal, 0, 0.0, vp(dq), dq.stride(0), dq.stride(1), vp(dk), dk.stride(0), dk.stride(1),
        vp(dv), dv.stride(0), dv.stride(1), vp(wsb), ws_bytes,
        ctypes.c_void_p(_lib.status_word(dev).data_ptr()), ctypes.c_void_p(_lib.stream_ptr(dev)))
    _lib.check(rc, "gko_fmha_varlen_bwd")
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    _check((dq, dk, dv), ref)
    for buf, n in ((bq, t * hq * d), (bk, t * hkv * d), (bv, t * hkv * d)):
        assert (buf[n:] == canary).all()
    assert (wsb[ws_bytes // 4:] == canary).all()
