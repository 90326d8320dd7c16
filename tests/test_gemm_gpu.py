"""Parity of the tensor-core GEMM operators (addmm+GELU/ReLU, SwiGLU, down
projection) and the fp32 path against the CPU oracle, through the C ABI.

Tolerances (from the operator contract): bf16/fp16 outputs need
max|err| / max|ref| <= 2e-2 against the fp32 oracle; fp32 outputs need
max|err| / max|ref| <= 1e-3 with TF32 disabled.
"""

import pytest
import torch

import oracle
from evocompile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
F32_TOL = 1e-3


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return g


def _randn(g, *shape, std=1.0, dtype=torch.float32):
    return (torch.randn(*shape, generator=g) * std).to(dtype)


def _status_clean():
    assert _lib.read_status(torch.device("cuda", 0)) == 0, "a kernel reported a timeout"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    "m,n,k",
    [(128, 256, 64), (256, 512, 128), (200, 264, 72), (1, 8, 8), (77, 1000, 520), (1024, 768, 1024)],
)
@pytest.mark.parametrize("b_layout", ["wt_view", "kn_contig"])
def test_addmm_gelu(dtype, m, n, k, b_layout):
    g = _gen(1000 + m + n + k)
    x = _randn(g, m, k, dtype=dtype)
    w = _randn(g, n, k, std=k ** -0.5, dtype=dtype)
    b = _randn(g, n, std=0.02, dtype=dtype)
    ref = oracle.addmm_gelu(b, x, w.t())
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    mat2 = wd.t() if b_layout == "wt_view" else wd.t().contiguous()
    out = ops.addmm_act(bd, xd, mat2, _lib.ACT_GELU)
    torch.cuda.synchronize()
    _status_clean()
    assert out.shape == (m, n) and out.dtype == dtype
    assert oracle.rel_err(out, ref) <= BF16_TOL


@pytest.mark.parametrize("act", [_lib.ACT_NONE, _lib.ACT_RELU])
def test_addmm_other_epilogues(act):
    g = _gen(7)
    x = _randn(g, 300, 256, dtype=torch.bfloat16)
    w = _randn(g, 384, 256, std=1 / 16, dtype=torch.bfloat16)
    b = _randn(g, 384, std=0.02, dtype=torch.float32)
    ref = oracle.addmm_act(b, x, w.t(), {0: "none", 2: "relu"}[act])
    out = ops.addmm_act(b.cuda(), x.cuda(), w.cuda().t(), act)
    torch.cuda.synchronize()
    assert oracle.rel_err(out, ref) <= BF16_TOL


def test_addmm_gelu_3d_input():
    g = _gen(11)
    x = _randn(g, 4, 33, 128, dtype=torch.bfloat16)
    w = _randn(g, 96, 128, std=128 ** -0.5, dtype=torch.bfloat16)
    b = _randn(g, 96, std=0.02, dtype=torch.bfloat16)
    ref = oracle.addmm_gelu(b, x, w.t())
    out = ops.addmm_act(b.cuda(), x.cuda(), w.cuda().t())
    assert out.shape == (4, 33, 96)
    assert oracle.rel_err(out, ref) <= BF16_TOL


def test_addmm_gelu_fp32_config():
    """GEMM+bias+GELU fp32: X[512,1024] ~ N(0,1), W[4096,1024] ~ N(0,1/1024), b ~ N(0,0.02)."""
    gx, gw, gb = _gen(0), _gen(1), _gen(2)
    x = torch.randn(512, 1024, generator=gx)
    w = torch.randn(4096, 1024, generator=gw) * (1024 ** -0.5)
    b = torch.randn(4096, generator=gb) * 0.02
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = oracle.addmm_gelu(b, x, w.t())
        out = ops.addmm_act(b.cuda(), x.cuda(), w.cuda().t())
        torch.cuda.synchronize()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert out.dtype == torch.float32
    assert oracle.rel_err(out, ref) <= F32_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,h,k", [(128, 128, 64), (256, 384, 256), (130, 200, 72), (1, 8, 16), (513, 1024, 512)])
@pytest.mark.parametrize("w_layout", ["row", "transposed_view"])
def test_gemm_swiglu(dtype, m, h, k, w_layout):
    g = _gen(2000 + m + h + k)
    x = _randn(g, m, k, dtype=dtype)
    w = _randn(g, 2 * h, k, std=k ** -0.5, dtype=dtype)
    ref = oracle.gemm_swiglu(x, w)
    wd = w.cuda() if w_layout == "row" else w.t().contiguous().cuda().t()
    out = ops.linear_swiglu(x.cuda(), wd)
    torch.cuda.synchronize()
    _status_clean()
    assert out.shape == (m, h)
    assert oracle.rel_err(out, ref) <= BF16_TOL


def test_gemm_swiglu_fp32():
    g = _gen(5)
    x = _randn(g, 3, 50, 64)
    w = _randn(g, 2 * 72, 64, std=1 / 8)
    ref = oracle.gemm_swiglu(x, w)
    out = ops.linear_swiglu(x.cuda(), w.cuda())
    assert out.shape == (3, 50, 72)
    assert oracle.rel_err(out, ref) <= F32_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(300, 264, 256), (1, 8, 64), (129, 520, 128), (256, 512, 1024)])
@pytest.mark.parametrize("in_place", [False, True])
def test_linear_residual(dtype, m, n, k, in_place):
    """x @ w^T + r with the residual add in the GEMM epilogue, also in place (out is r)."""
    g = _gen(m + n + k + int(in_place))
    x = _randn(g, m, k, dtype=dtype)
    w = _randn(g, n, k, std=k ** -0.5, dtype=dtype)
    r = _randn(g, m, n, dtype=dtype)
    ref = x.float() @ w.float().t() + r.float()
    rd = r.cuda()
    out = ops.linear_residual(x.cuda(), w.cuda(), rd, out=rd if in_place else None)
    assert out.shape == (m, n) and out.dtype == dtype
    if in_place:
        assert out.data_ptr() == rd.data_ptr()
    _status_clean()
    assert oracle.rel_err(out, ref) <= BF16_TOL


def test_swiglu_mlp_small():
    g = _gen(9)
    x = _randn(g, 256, 512, dtype=torch.bfloat16)
    wgu = _randn(g, 2 * 1024, 512, std=0.02, dtype=torch.bfloat16)
    wd = _randn(g, 512, 1024, std=0.02, dtype=torch.bfloat16)
    ref = oracle.swiglu_mlp(x, wgu, wd)
    out = ops.swiglu_mlp(x.cuda(), wgu.cuda(), wd.cuda())
    assert oracle.rel_err(out, ref) <= BF16_TOL


@pytest.mark.slow
def test_swiglu_mlp_full_config_sampled_rows():
    """SwiGLU MLP at the Llama-3-8B shape (X[8192,4096], Wg/Wu[14336,4096], Wdown[4096,14336]);
    the fp32 oracle is evaluated on 192 sampled token rows (rows are independent)."""
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    x = torch.randn(8192, 4096, device=dev).to(torch.bfloat16)
    wgu = (torch.randn(2 * 14336, 4096, device=dev) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(4096, 14336, device=dev) * 0.02).to(torch.bfloat16)
    out = ops.swiglu_mlp(x, wgu, wd)
    torch.cuda.synchronize()
    _status_clean()
    rows = torch.randperm(8192, generator=_gen(3))[:192].to(dev)
    ref = oracle.swiglu_mlp(x[rows].cpu(), wgu.cpu(), wd.cpu())
    assert oracle.rel_err(out[rows], ref) <= BF16_TOL
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
def test_silu_mul(dtype, n):
    g = _gen(n)
    x = _randn(g, n, dtype=dtype)
    y = _randn(g, n, dtype=dtype)
    ref = oracle.silu_mul(x, y)
    out = ops.silu_mul(x.cuda(), y.cuda())
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert oracle.rel_err(out, ref) <= tol


def test_empty_inputs():
    dev = torch.device("cuda", 0)
    x = torch.empty(0, 64, device=dev, dtype=torch.bfloat16)
    w = torch.randn(128, 64, device=dev).to(torch.bfloat16)
    assert ops.addmm_act(None, x, w.t()).shape == (0, 128)
    assert ops.linear_swiglu(x, w).shape == (0, 64)


def test_rejects_unsupported():
    dev = torch.device("cuda", 0)
    x = torch.randn(16, 12, device=dev).to(torch.bfloat16)  # K % 8 != 0
    w = torch.randn(32, 12, device=dev).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiples of 8"):
        ops.addmm_act(None, x, w.t())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (264, 200, 1000), (8, 8, 16), (1000, 520, 77 * 8), (4096, 1024, 512),
                                   (528, 256, 300), (64, 72, 1)])
@pytest.mark.parametrize("b_layout", ["wt_view", "kn_contig"])
def test_weight_grad_transposed_mat1(dtype, m, n, k, b_layout):
    """dW = dZ^T X: mat1 is the transposed view of a row-major [k, m] tensor, read in place as
    an MN-major operand (no copy); ragged m, n and k."""
    if b_layout == "wt_view" and k % 8:
        pytest.skip("a K-major mat2 needs k % 8 == 0 (its rows are k elements)")
    g = _gen(m + n + k + (b_layout == "wt_view"))
    a_store = _randn(g, k, m, dtype=dtype)           # e.g. dZ [tokens, features]
    a = a_store.cuda().t()                            # [m, k], strides (1, m)
    if b_layout == "kn_contig":
        b_host = _randn(g, k, n, dtype=dtype)         # e.g. X [tokens, in]
        b = b_host.cuda()
    else:
        b_host = _randn(g, n, k, dtype=dtype).t()
        b = b_host.t().contiguous().cuda().t()
    out = ops.addmm_act(None, a, b, _lib.ACT_NONE)
    torch.cuda.synchronize()
    _status_clean()
    ref = a_store.float().t() @ b_host.float()
    assert out.shape == (m, n)
    assert oracle.rel_err(out, ref) <= BF16_TOL


def test_weight_grad_with_activation_is_refused():
    """The transposed-mat1 path has the plain epilogue only; with GELU the op copies mat1 to
    row-major first (same result), and the C ABI refuses the transposed form directly."""
    import ctypes

    a = torch.randn(64, 128, dtype=torch.bfloat16, device="cuda").t()
    b = torch.randn(64, 64, dtype=torch.bfloat16, device="cuda")
    ref = torch.nn.functional.gelu(a.float() @ b.float())
    assert oracle.rel_err(ops.addmm_act(None, a, b, _lib.ACT_GELU), ref.cpu()) <= BF16_TOL
    out = torch.empty(128, 64, dtype=torch.bfloat16, device="cuda")
    dev = torch.device("cuda", 0)
    rc = _lib.load().gko_addmm_act(
        _lib.BF16, _lib.ACT_GELU, 128, 64, 64, ctypes.c_void_p(a.data_ptr()), 1, 128, ctypes.c_void_p(b.data_ptr()),
        64, 1, ctypes.c_void_p(0), 0, ctypes.c_void_p(out.data_ptr()), 64,
        ctypes.c_void_p(_lib.status_word(dev).data_ptr()), ctypes.c_void_p(_lib.stream_ptr(dev)))
    assert rc == _lib.ERR_UNSUPPORTED and "transposed" in _lib.last_error()


def test_gemm_cta_cap_keeps_results():
    """A GEMM confined to a few SMs (gko_set_gemm_ctas) computes the same result; the cap is
    restored afterwards and a negative cap is refused."""
    g = _gen(91)
    x = _randn(g, 1000, 512, dtype=torch.bfloat16).cuda()
    w = _randn(g, 768, 512, std=512 ** -0.5, dtype=torch.bfloat16).cuda()
    full = ops.linear(x, w)
    prev = ops.set_gemm_ctas(7)
    try:
        capped = ops.linear(x, w)
    finally:
        assert ops.set_gemm_ctas(prev) == 7
    torch.cuda.synchronize()
    _status_clean()
    assert torch.equal(full, capped)
    with pytest.raises(RuntimeError, match="CTA limit"):
        ops.set_gemm_ctas(-1)


def test_gelu_epilogue_within_one_bf16_ulp():
    """The tensor-core epilogue's GELU (erf from Abramowitz & Stegun 7.1.26, |error| <= 1.5e-7) on
    exactly known pre-activations z (one-hot mat1 rows): every output is within one bf16 ulp of
    the exact-erf GELU of z rounded to bf16, or, in the negative tail where GELU is tiny and
    1 + erf cancels (for CUDA's erff too), within an absolute 2e-7 |z|."""
    z = torch.linspace(-8, 8, 4096).to(torch.bfloat16)
    m = z.numel()
    a = torch.zeros(m, 8, dtype=torch.bfloat16)
    a[:, 0] = z
    b = torch.zeros(8, 16, dtype=torch.bfloat16)
    b[0, :] = 1
    out = ops.addmm_act(None, a.cuda(), b.cuda(), _lib.ACT_GELU)
    torch.cuda.synchronize()
    _status_clean()
    exact = torch.nn.functional.gelu(z.double(), approximate="none")
    got = out[:, 0].cpu().double()
    ref = exact.to(torch.bfloat16).double()
    ulp = torch.maximum(ref.abs(), torch.full_like(ref, 2 ** -126)) * 2 ** -7
    assert ((got - ref).abs() <= ulp + 2e-7 * z.double().abs() + 1e-30).all()
    assert torch.equal(out[:, 0], out[:, 15])
