"""The drop-in path on the GPU, as the reference harness uses it: register catalog kernels, compile a model
with torch.compile (Inductor) so the FX passes land the gko ops, run a training step, and check the loss
against eager with the reference Evaluator's rule abs(c - b) <= 1e-2 + 1e-2 |b| (agent/metrics.py:19-57)."""

import pytest
import torch
import torch.nn.functional as F

from evocompile_b200 import kernels

pytestmark = pytest.mark.gpu


def _loss_consistent(b, c, atol=1e-2, rtol=1e-2):
    return abs(c - b) <= atol + rtol * abs(b)


class _MLP(torch.nn.Module):
    def __init__(self, d=256, h=1024):
        super().__init__()
        self.fc1 = torch.nn.Linear(d, h)
        self.fc2 = torch.nn.Linear(h, d)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x)))


class _Attn(torch.nn.Module):
    """An attention block that calls the hook target the way the reference's rewrites do."""

    def __init__(self, d=256, heads=4):
        super().__init__()
        self.h, self.dh = heads, d // heads
        self.qkv = torch.nn.Linear(d, 3 * d)
        self.o = torch.nn.Linear(d, d)

    def forward(self, x, attn):
        B, S, d = x.shape
        q, k, v = self.qkv(x).view(B, S, 3, self.h, self.dh).unbind(2)
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        y = attn(q, k, v, None, self.dh ** -0.5, 1)
        return self.o(y.transpose(1, 2).reshape(B, S, d))


def _train_step(model, x, *extra):
    out = model(x, *extra)
    loss = out.float().square().mean()
    loss.backward()
    return float(loss)


@pytest.fixture(autouse=True)
def _clean():
    kernels.reset_installed()
    torch._dynamo.reset()
    yield
    kernels.reset_installed()
    torch._dynamo.reset()


def test_compiled_linear_gelu_lands_on_gko_op_and_matches_eager():
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    model = _MLP().to(dev).to(torch.bfloat16)
    x = torch.randn(8, 64, 256, device=dev, dtype=torch.bfloat16)
    ref = _train_step(model, x)
    model.zero_grad()
    kernels.register("addmm_gelu")
    calls = {"n": 0}
    orig = kernels.addmm_gelu._addmm_gelu_forward

    def counting(*a):
        calls["n"] += 1
        return orig(*a)

    kernels.addmm_gelu._addmm_gelu_forward = counting
    try:
        compiled = torch.compile(model)
        got = _train_step(compiled, x)
    finally:
        kernels.addmm_gelu._addmm_gelu_forward = orig
    assert calls["n"] >= 1, "the compiled graph did not call gko::addmm_gelu"
    assert _loss_consistent(ref, got), (ref, got)
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_attention_hook_training_step_matches_eager():
    torch.manual_seed(1)
    dev = torch.device("cuda", 0)
    model = _Attn().to(dev).to(torch.bfloat16)
    x = torch.randn(2, 128, 256, device=dev, dtype=torch.bfloat16)

    def sdpa(q, k, v, bias, scale, causal):
        return F.scaled_dot_product_attention(q, k, v, scale=scale, is_causal=bool(causal))

    ref = _train_step(model, x, sdpa)
    grads_ref = [p.grad.clone() for p in model.parameters()]
    model.zero_grad()
    kernels.register("fused_sdpa")
    attn = kernels.attn_call()
    got = _train_step(torch.compile(model), x, attn)
    assert _loss_consistent(ref, got), (ref, got)
    for g0, p in zip(grads_ref, model.parameters()):
        assert (p.grad.float() - g0.float()).abs().max() <= 5e-2 * g0.float().abs().max() + 1e-3


def test_gemm_swiglu_apply_autograd():
    torch.manual_seed(2)
    dev = torch.device("cuda", 0)
    kernels.register("gemm_swiglu")
    x = torch.randn(64, 256, device=dev, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(2 * 512, 256, device=dev) * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = kernels.gemm_swiglu.apply(x, w)
    y.float().square().mean().backward()
    gx, gw = x.grad.clone(), w.grad.clone()
    x.grad = w.grad = None
    gu = F.linear(x, w)
    g, u = gu.chunk(2, -1)
    (F.silu(g) * u).float().square().mean().backward()
    assert (gx.float() - x.grad.float()).abs().max() <= 3e-2 * x.grad.float().abs().max()
    assert (gw.float() - w.grad.float()).abs().max() <= 3e-2 * w.grad.float().abs().max()
