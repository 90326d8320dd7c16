"""Training forms of the GEMM operators (forward kernels that also write the pre-activation,
backward without recomputing the forward GEMM): forward outputs identical to the plain
kernels', pre-activations and gradients against fp32 autograd of the oracle.
bf16: max|err| / max|ref| <= 2e-2."""

import pytest
import torch

import oracle
from evocompile_b200 import _lib, ops
from evocompile_b200.kernels import addmm_gelu, gemm_swiglu

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _grads_oracle(fn, *args):
    ts = [a.detach().float().cpu().requires_grad_(True) for a in args]
    out = fn(*ts)
    return out, ts


@pytest.mark.parametrize("lead", [(300,), (2, 129)])
def test_addmm_gelu_aux_forward(lead):
    g = torch.Generator().manual_seed(len(lead))
    K, N = 256, 520
    x = torch.randn(*lead, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).cuda()
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    out, z = ops.addmm_act(b, x, w.t(), _lib.ACT_GELU, save_pre=True)
    plain = ops.addmm_act(b, x, w.t(), _lib.ACT_GELU)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
    assert oracle.rel_err(z, oracle.addmm_act(b, x, w.t(), "none")) <= TOL


def test_addmm_gelu_train_backward():
    g = torch.Generator().manual_seed(3)
    M, K, N = 300, 256, 520
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    xd, wd, bd = (t.cuda().requires_grad_(True) for t in (x, w, b))
    y = addmm_gelu.addmm_gelu_train(bd, xd, wd.t())
    y.backward(dy.cuda())
    ref_y, (rb, rx, rw) = _grads_oracle(lambda bb, xx, ww: oracle.addmm_gelu(bb, xx, ww.t()), b, x, w)
    ref_y.backward(dy.float())
    assert oracle.rel_err(y, ref_y) <= TOL
    assert oracle.rel_err(xd.grad, rx.grad) <= TOL
    assert oracle.rel_err(wd.grad, rw.grad) <= TOL
    assert oracle.rel_err(bd.grad, rb.grad) <= TOL
    assert _lib.read_status(torch.device("cuda", 0)) == 0


@pytest.mark.parametrize("lead", [(300,), (3, 77)])
def test_gemm_swiglu_aux_forward(lead):
    g = torch.Generator().manual_seed(10 + len(lead))
    D, H = 256, 264
    x = torch.randn(*lead, D, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(2 * H, D, generator=g) * D ** -0.5).to(torch.bfloat16).cuda()
    out, gu = ops.linear_swiglu(x, w, save_pre=True)
    plain = ops.linear_swiglu(x, w)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
    ref_gu = torch.nn.functional.linear(x.float().cpu(), w.float().cpu())
    assert gu.shape == ref_gu.shape
    assert oracle.rel_err(gu, ref_gu) <= TOL


def test_aux_outputs_many_tiles():
    """512 output tiles on at most 148 persistent CTAs, so every CTA converts several tiles and
    reuses its staging buffer and both accumulators: the GELU pre-activation equals the plain
    (no activation) GEMM bit for bit (same accumulation, same bias add), and the SwiGLU
    gate / up pre-activations match an fp32 GEMM."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(21)
    M, K, N = 4096, 256, 4096
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
    b = (torch.randn(N, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    out, z = ops.addmm_act(b, x, w.t(), _lib.ACT_GELU, save_pre=True)
    plain = ops.addmm_act(b, x, w.t(), _lib.ACT_GELU)
    pre = ops.addmm_act(b, x, w.t(), _lib.ACT_NONE)
    H = 2048
    y, gu = ops.linear_swiglu(x, w, save_pre=True)  # w = [Wg; Wu], H = N / 2
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    assert torch.equal(out, plain)
    assert torch.equal(z, pre)
    ref = x.float() @ w.float().t()
    assert gu.shape == (M, 2 * H)
    assert oracle.rel_err(gu.cpu(), ref.cpu()) <= 1e-2
    assert torch.equal(y, ops.linear_swiglu(x, w))


def test_swiglu_bwd_kernel():
    g = torch.Generator().manual_seed(5)
    R, H = 333, 136
    gu = torch.randn(R, 2 * H, generator=g).to(torch.bfloat16)
    dy = torch.randn(R, H, generator=g).to(torch.bfloat16)
    got = ops.swiglu_bwd(dy.cuda(), gu.cuda())
    gf, uf = gu.float()[:, :H], gu.float()[:, H:]
    s = torch.sigmoid(gf)
    ref = torch.cat([dy.float() * uf * s * (1 + gf * (1 - s)), dy.float() * gf * s], dim=1)
    assert oracle.rel_err(got, ref) <= TOL


def test_gemm_swiglu_train_backward():
    g = torch.Generator().manual_seed(7)
    M, D, H = 300, 256, 264
    x = torch.randn(M, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * H, D, generator=g) * D ** -0.5).to(torch.bfloat16)
    dy = torch.randn(M, H, generator=g).to(torch.bfloat16)
    xd, wd = (t.cuda().requires_grad_(True) for t in (x, w))
    y = gemm_swiglu.apply_train(xd, wd)
    y.backward(dy.cuda())
    ref_y, (rx, rw) = _grads_oracle(oracle.gemm_swiglu, x, w)
    ref_y.backward(dy.float())
    assert oracle.rel_err(y, ref_y) <= TOL
    assert oracle.rel_err(xd.grad, rx.grad) <= TOL
    assert oracle.rel_err(wd.grad, rw.grad) <= TOL
    assert _lib.read_status(torch.device("cuda", 0)) == 0


def test_train_forms_reject_fp32():
    x = torch.randn(16, 32, device="cuda")
    w = torch.randn(64, 32, device="cuda")
    with pytest.raises(RuntimeError, match="bf16 / f16"):
        ops.linear_swiglu(x, w, save_pre=True)
