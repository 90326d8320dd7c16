"""Parity of the tcgen05 attention forward against the CPU oracle (fp32),
through the C ABI. bf16/fp16 outputs: max|err| / max|ref| <= 2e-2; lse is
compared with an absolute tolerance of 2e-2 on rows that have unmasked keys.
"""

import pytest
import torch

import oracle
from evocompile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _qkv(seed, z, hq, hkv, sq, sk, d, dtype, layout="bhsd"):
    g = torch.Generator().manual_seed(seed)
    if layout == "bhsd":
        q = torch.randn(z, hq, sq, d, generator=g).to(dtype)
        k = torch.randn(z, hkv, sk, d, generator=g).to(dtype)
        v = torch.randn(z, hkv, sk, d, generator=g).to(dtype)
        return q, k, v, (lambda t: t.cuda())
    # [z, s, h, d] storage viewed as [z, h, s, d]
    q = torch.randn(z, sq, hq, d, generator=g).to(dtype).transpose(1, 2)
    k = torch.randn(z, sk, hkv, d, generator=g).to(dtype).transpose(1, 2)
    v = torch.randn(z, sk, hkv, d, generator=g).to(dtype).transpose(1, 2)
    return q, k, v, (lambda t: t.transpose(1, 2).contiguous().cuda().transpose(1, 2))


def _check(out, lse, ref_out, ref_lse):
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0, "a kernel reported a timeout"
    assert oracle.rel_err(out, ref_out) <= TOL
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    if fin.any():
        assert (lse.cpu()[fin] - ref_lse[fin]).abs().max().item() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("s", [1, 63, 128, 200, 513])
def test_fmha_dense(dtype, d, causal, s):
    q, k, v, dev = _qkv(s * 10 + d + causal, 2, 3, 3, s, s, d, dtype)
    ref_o, ref_l = oracle.attention(q, k, v, None, d ** -0.5, causal)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), None, d ** -0.5, causal)
    assert out.shape == q.shape and lse.shape == (2 * 3, s)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
def test_fmha_growing_logits(d, causal):
    """Key norms grow with each 128-key tile and query norms differ per row, so the row
    maximum of later tiles exceeds the running maximum by more than the lazy-rescale
    threshold for some rows of a warp and not for others: covers the first-half recompute,
    the O rescale and the rows that keep their maximum."""
    g = torch.Generator().manual_seed(77 + d + causal)
    sq, sk = 256, 640
    q = torch.randn(1, 2, sq, d, generator=g) * (0.1 + 2 * torch.rand(1, 2, sq, 1, generator=g))
    grow = 1.0 + 3.0 * (torch.arange(sk) // 128).float()
    k = torch.randn(1, 2, sk, d, generator=g) * grow.view(1, 1, sk, 1)
    v = torch.randn(1, 2, sk, d, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    ref_o, ref_l = oracle.attention(q, k, v, None, d ** -0.5, causal)
    out, lse = ops.fmha_fwd(q.cuda(), k.cuda(), v.cuda(), None, d ** -0.5, causal)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("sq,sk", [(64, 300), (300, 64), (129, 1000)])
@pytest.mark.parametrize("causal", [0, 1])
def test_fmha_cross_lengths(sq, sk, causal):
    q, k, v, dev = _qkv(sq + sk, 1, 2, 2, sq, sk, 128, torch.bfloat16)
    ref_o, ref_l = oracle.attention(q, k, v, None, 0.1, causal)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), None, 0.1, causal)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("hq,hkv", [(8, 2), (8, 1), (4, 4)])
def test_fmha_gqa_bshd_layout(hq, hkv):
    q, k, v, dev = _qkv(hq * 7 + hkv, 2, hq, hkv, 300, 300, 128, torch.bfloat16, layout="bshd")
    ref_o, ref_l = oracle.attention(q, k, v, None, 128 ** -0.5, 1)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), None, 128 ** -0.5, 1)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("kind", ["keypad", "keypad4d", "full", "full_bcast", "swin"])
def test_fmha_bias(kind):
    z, h, s, d = 4, 2, 150, 64
    q, k, v, dev = _qkv(31, z, h, h, s, s, d, torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    if kind == "keypad":
        bias = torch.zeros(z, s)
        bias[:, -20:] = torch.finfo(torch.bfloat16).min
        bias = bias.to(torch.bfloat16)
    elif kind == "keypad4d":
        bias = (torch.randn(z, 1, 1, s, generator=g)).to(torch.bfloat16)
    elif kind == "full":
        bias = torch.randn(z, h, s, s, generator=g).to(torch.float32)
    elif kind == "full_bcast":
        bias = torch.randn(1, 1, s, s, generator=g).to(torch.bfloat16)
    else:
        bias = torch.randn(2, h, s, s, generator=g).to(torch.bfloat16)  # nW = 2 windows, z = 2 * nW
    ref_o, ref_l = oracle.attention(q, k, v, bias, 0.125, 0)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), bias.cuda(), 0.125, 0)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("window,causal,softcap", [(32, 0, 0.0), (100, 1, 0.0), (0, 1, 30.0), (50, 0, 5.0)])
def test_fmha_window_softcap(window, causal, softcap):
    q, k, v, dev = _qkv(window + causal, 2, 2, 2, 400, 400, 128, torch.bfloat16)
    ref_o, ref_l = oracle.attention(q, k, v, None, 128 ** -0.5, causal, window, softcap)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), None, 128 ** -0.5, causal, window, softcap)
    _check(out, lse, ref_o, ref_l)


def test_fmha_fully_masked_rows():
    """Batch 0 has every key masked (-inf key padding): zeros out, lse = -inf."""
    z, h, s, d = 2, 2, 70, 64
    q, k, v, dev = _qkv(3, z, h, h, s, s, d, torch.bfloat16)
    bias = torch.zeros(z, s)
    bias[0, :] = float("-inf")
    ref_o, ref_l = oracle.attention(q, k, v, bias, 0.125, 0)
    out, lse = ops.fmha_fwd(dev(q), dev(k), dev(v), bias.cuda(), 0.125, 0)
    _check(out, lse, ref_o, ref_l)
    assert out[0].abs().max().item() == 0.0


@pytest.mark.parametrize("causal", [0, 1])
@pytest.mark.parametrize("hq,hkv", [(8, 2), (4, 4)])
def test_fmha_varlen(causal, hq, hkv):
    lens = [1, 65, 300, 128, 7, 513]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    t = int(cu[-1])
    g = torch.Generator().manual_seed(len(lens) + hq)
    q = torch.randn(t, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(t, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(t, hkv, 128, generator=g).to(torch.bfloat16)
    ref_o, ref_l = oracle.attention_varlen(q, k, v, cu, cu, 128 ** -0.5, causal)
    out, lse = ops.fmha_varlen_fwd(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), cu.cuda(), max(lens), max(lens),
                                   128 ** -0.5, causal)
    _check(out, lse, ref_o, ref_l)


@pytest.mark.slow
def test_fmha_full_config_sampled_heads():
    """Causal FMHA at B=8, H=32, S=4096, D=128 in [B,S,H,D] layout; the fp32 oracle
    checks three (batch, head) slices."""
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    B, S, H, D = 8, 4096, 32, 128
    qs = torch.randn(B, S, H, D, device=dev).to(torch.bfloat16)
    ks = torch.randn(B, S, H, D, device=dev).to(torch.bfloat16)
    vs = torch.randn(B, S, H, D, device=dev).to(torch.bfloat16)
    q, k, v = qs.transpose(1, 2), ks.transpose(1, 2), vs.transpose(1, 2)
    out, lse = ops.fmha_fwd(q, k, v, None, D ** -0.5, 1)
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    for b, h in [(0, 0), (3, 17), (7, 31)]:
        ro, rl = oracle.attention(q[b:b + 1, h:h + 1].cpu(), k[b:b + 1, h:h + 1].cpu(),
                                  v[b:b + 1, h:h + 1].cpu(), None, D ** -0.5, 1)
        assert oracle.rel_err(out[b:b + 1, h:h + 1], ro) <= TOL
        assert (lse.view(B, H, S)[b, h].cpu() - rl.view(S)).abs().max().item() <= 2e-2


@pytest.mark.slow
def test_fmha_varlen_full_config():
    """The benchmarked GQA varlen configuration exactly: 16 sequences with lengths drawn by
    randint(512, 8193) from seed 0, Hq=64, Hkv=8, D=128, causal. The fp32 oracle checks every
    head of the shortest and the longest sequence and four more (sequence, head) pairs."""
    gl = torch.Generator().manual_seed(0)
    lens = torch.randint(512, 8193, (16,), generator=gl).tolist()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    t = int(cu[-1])
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4000)
    q = torch.randn(t, 64, 128, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(t, 8, 128, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(t, 8, 128, device=dev, generator=g).to(torch.bfloat16)
    cud = cu.to(dev)
    out, lse = ops.fmha_varlen_fwd(q, k, v, cud, cud, max(lens), max(lens), 128 ** -0.5, 1)
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    short, long_ = min(range(16), key=lambda i: lens[i]), max(range(16), key=lambda i: lens[i])
    pairs = [(short, h) for h in range(64)] + [(long_, h) for h in range(64)]
    rnd = torch.Generator().manual_seed(1)
    pairs += [(int(torch.randint(16, (1,), generator=rnd)), int(torch.randint(64, (1,), generator=rnd)))
              for _ in range(4)]
    for sq, h in pairs:
        a, b = int(cu[sq]), int(cu[sq + 1])
        hk = h // 8
        qs = q[a:b, h].cpu()[None, None]
        ks = k[a:b, hk].cpu()[None, None]
        vs = v[a:b, hk].cpu()[None, None]
        ro, rl = oracle.attention(qs, ks, vs, None, 128 ** -0.5, 1)
        assert oracle.rel_err(out[a:b, h], ro[0, 0]) <= TOL, (sq, h)
        assert (lse[h, a:b].cpu() - rl.view(-1)).abs().max().item() <= 2e-2, (sq, h)
