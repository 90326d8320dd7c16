"""The drop-in boundary on CPU: the catalog registers the reference's op names
and schemas, fake implementations give the reference's output shapes, the FX
passes rewrite the same graph patterns, and a compiled graph calls the gko op
(proved by the op refusing CPU tensors: there is no CPU fallback)."""

import pytest
import torch
import torch.nn.functional as F
from torch.fx.experimental.proxy_tensor import make_fx
from torch._subclasses.fake_tensor import FakeTensorMode

from evocompile_b200 import kernels
from evocompile_b200.kernels import addmm_gelu, silu_mul, pass_install

EXPECTED_SCHEMAS = {
    # reference: eval/kernels/addmm_gelu.py:197-201, gemm_swiglu.py:213-215, fused_sdpa.py:912-922,947-960,981-989,
    # cutlass_gemm_attn.py:87-97, silu_mul.py:71-73
    "addmm_gelu": "gko::addmm_gelu(Tensor bias, Tensor mat1, Tensor mat2) -> Tensor",
    "gemm_swiglu": "gko::gemm_swiglu(Tensor x, Tensor weight) -> Tensor",
    "fused_sdpa_pair": "gko::fused_sdpa_pair(Tensor q, Tensor k, Tensor v, Tensor attn_bias, float scale, SymInt causal, SymInt window, float softcap) -> (Tensor, Tensor)",
    "fused_sdpa_bwd": "gko::fused_sdpa_bwd(Tensor q, Tensor k, Tensor v, Tensor attn_bias, Tensor out, Tensor lse, Tensor dout, float scale, SymInt causal, SymInt window, float softcap) -> (Tensor, Tensor, Tensor)",
    "fused_sdpa": "gko::fused_sdpa(Tensor q, Tensor k, Tensor v, Tensor attn_bias, float scale, SymInt causal) -> Tensor",
    "cutlass_fmha_pair": "gko::cutlass_fmha_pair(Tensor q, Tensor k, Tensor v, Tensor attn_bias, float scale, SymInt causal, SymInt window, float softcap) -> (Tensor, Tensor)",
    "silu_mul": "gko::silu_mul(Tensor x, Tensor y) -> Tensor",
}


@pytest.fixture(autouse=True)
def _registered():
    kernels.reset_installed()
    for name in ("addmm_gelu", "gemm_swiglu", "fused_sdpa", "silu_mul"):
        kernels.register(name)
    from evocompile_b200.kernels import cutlass_gemm_attn

    cutlass_gemm_attn._ensure_op()
    yield
    kernels.reset_installed()


def test_catalog_and_register_idempotent():
    assert set(kernels.list_kernels()) >= {"addmm_gelu", "gemm_swiglu", "fused_sdpa", "silu_mul"}
    assert "already registered" in kernels.register("addmm_gelu")
    assert kernels.attn_call() is kernels.fused_sdpa.fused_attention
    with pytest.raises(ValueError, match="unknown kernel"):
        kernels.register("no_such_kernel")


def test_schemas_match_reference():
    for name, schema in EXPECTED_SCHEMAS.items():
        assert str(getattr(torch.ops.gko, name).default._schema) == schema


def test_reset_installed_clears_passes():
    import torch._inductor.config as cfg

    assert cfg.pre_grad_custom_pass is not None and cfg.post_grad_custom_pre_pass is not None
    kernels.reset_installed()
    assert cfg.pre_grad_custom_pass is None and cfg.post_grad_custom_pre_pass is None
    assert kernels.attn_call() is None


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(4, 9, 64)
        w = torch.empty(96, 64)
        assert torch.ops.gko.addmm_gelu(torch.empty(96), x, w.t()).shape == (4, 9, 96)
        assert torch.ops.gko.gemm_swiglu(x, torch.empty(256, 64)).shape == (4, 9, 128)
        q = torch.empty(2, 8, 100, 64).transpose(1, 2)  # strided view in
        out, lse = torch.ops.gko.fused_sdpa_pair(q, q, q, torch.empty(0), 0.1, 1, 0, 0.0)
        assert out.shape == q.shape and out.is_contiguous() and lse.shape == (2 * 100, 8)
        assert lse.dtype == torch.float32
        o2, l2 = torch.ops.gko.fmha_varlen_fwd(torch.empty(50, 8, 128), torch.empty(50, 2, 128),
                                               torch.empty(50, 2, 128), torch.empty(3, dtype=torch.int32),
                                               torch.empty(3, dtype=torch.int32), 30, 30, 0.1, 1)
        assert o2.shape == (50, 8, 128) and l2.shape == (8, 50)


def test_ops_refuse_cpu_tensors():
    x = torch.randn(4, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.gko.addmm_gelu(torch.zeros(8), x, torch.randn(16, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.gko.gemm_swiglu(x, torch.randn(8, 16))
    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.gko.fused_sdpa_pair(q, q, q, torch.empty(0), 0.1, 0, 0, 0.0)


def test_norm_ops_refuse_mismatched_residual_and_weight():
    """The RMSNorm kernels read a residual of x's shape and a weight of x's last dim in x's dtype;
    anything else is refused on the host before a launch could read out of bounds."""
    from evocompile_b200 import ops

    x = torch.zeros(6, 64, dtype=torch.bfloat16)
    ops._check_norm_args("rms_stats", x, torch.zeros_like(x))
    ops._check_norm_args("rmsnorm", x, None, torch.ones(64, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="residual"):
        ops._check_norm_args("rms_stats", x, torch.zeros(5, 64, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="residual"):
        ops._check_norm_args("rms_stats", x, torch.zeros(6, 64, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="weight"):
        ops._check_norm_args("rmsnorm", x, None, torch.ones(32, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="weight"):
        ops._check_norm_args("rmsnorm", x, None, torch.ones(64, dtype=torch.float32))
    # rope_ checks the positions length before it reaches the device check
    with pytest.raises(RuntimeError, match="positions"):
        ops.rope_(torch.zeros(4, 2, 64).as_strided((4, 2, 64), (128, 64, 1)), positions=torch.zeros(3))


def _count(gm, op):
    return sum(1 for n in gm.graph.nodes if n.target == op)


class _LinearGelu(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.fc = torch.nn.Linear(16, 32)

    def forward(self, x):
        return F.gelu(self.fc(x))


def test_pass_rewrites_linear_module():
    gm = torch.fx.symbolic_trace(_LinearGelu())
    assert addmm_gelu.fuse_addmm_gelu(gm.graph) == 1
    gm.recompile()
    assert _count(gm, torch.ops.gko.addmm_gelu.default) == 1


@pytest.mark.parametrize("variant", ["addmm", "linear", "mm_add", "decomposed", "view_wrapped", "tanh_gelu"])
def test_pass_patterns(variant):
    def f(x, w, b):
        if variant == "addmm":
            return F.gelu(torch.addmm(b, x, w.t()))
        if variant == "linear":
            return F.gelu(F.linear(x, w, b))
        if variant == "mm_add":
            return F.gelu(torch.mm(x, w.t()) + b)
        if variant == "decomposed":
            z = torch.addmm(b, x, w.t())
            return z * 0.5 * (1.0 + torch.erf(z * 0.7071067811865476))
        if variant == "view_wrapped":
            return F.gelu(torch.addmm(b, x, w.t()).view(2, 2, 32))
        return F.gelu(torch.addmm(b, x, w.t()), approximate="tanh")

    gm = make_fx(f)(torch.randn(4, 16), torch.randn(32, 16), torch.randn(32))
    if variant == "decomposed":
        # make the graph look like decomposed pre-grad aten: mul(z, 0.5), mul(z, c) -> erf -> add 1 -> mul
        g = torch.fx.Graph()
        x, w, b = g.placeholder("x"), g.placeholder("w"), g.placeholder("b")
        wt = g.call_function(torch.ops.aten.t.default, (w,))
        z = g.call_function(torch.ops.aten.addmm.default, (b, x, wt))
        half = g.call_function(torch.ops.aten.mul.Tensor, (z, 0.5))
        sc = g.call_function(torch.ops.aten.mul.Tensor, (z, 0.7071067811865476))
        er = g.call_function(torch.ops.aten.erf.default, (sc,))
        one = g.call_function(torch.ops.aten.add.Tensor, (er, 1.0))
        out = g.call_function(torch.ops.aten.mul.Tensor, (half, one))
        g.output(out)
        gm = torch.fx.GraphModule(torch.nn.Module(), g)
    n = addmm_gelu.fuse_addmm_gelu(gm.graph)
    gm.recompile()
    if variant == "tanh_gelu":
        assert n == 0  # only the exact erf GELU is fused
    else:
        assert n == 1 and _count(gm, torch.ops.gko.addmm_gelu.default) == 1
        remaining = {str(nd.target) for nd in gm.graph.nodes if nd.op == "call_function"}
        assert "aten.gelu.default" not in remaining and "aten.erf.default" not in remaining


def test_pass_skips_when_preactivation_is_reused():
    def f(x, w, b):
        z = torch.addmm(b, x, w.t())
        return F.gelu(z) + z

    gm = make_fx(f)(torch.randn(4, 16), torch.randn(32, 16), torch.randn(32))
    assert addmm_gelu.fuse_addmm_gelu(gm.graph) == 0


def test_silu_mul_pass():
    def f(a, b):
        return F.silu(a) * b

    gm = make_fx(f)(torch.randn(8), torch.randn(8))
    assert silu_mul.fuse_silu_mul(gm.graph) == 1
    gm.recompile()
    assert _count(gm, torch.ops.gko.silu_mul.default) == 1


def test_compiled_graph_lands_on_gko_op():
    """Under torch.compile (Inductor, CPU) the installed pre-grad pass rewrites Linear+GELU to
    gko::addmm_gelu; running it on CPU tensors then reaches the op, which refuses them."""
    torch._dynamo.reset()
    model = _LinearGelu()
    compiled = torch.compile(model)
    with pytest.raises(Exception, match="CUDA"):
        compiled(torch.randn(3, 16))
    torch._dynamo.reset()


def test_pass_install_idempotent_and_composed():
    import torch._inductor.config as cfg

    kernels.reset_installed()
    calls = []
    p1 = lambda g: calls.append(1)  # noqa: E731
    p2 = lambda g: calls.append(2)  # noqa: E731
    pass_install.install_inductor_pass("post_grad_custom_pre_pass", p1, key="a")
    pass_install.install_inductor_pass("post_grad_custom_pre_pass", p1, key="a")
    pass_install.install_post_grad_pass(p2, key="b")
    cfg.post_grad_custom_pre_pass(torch.fx.Graph())
    assert calls == [1, 2]
    with pytest.raises(TypeError):
        pass_install.install_inductor_pass("pre_grad_custom_pass", 3)


def test_linear_residual_rejects_out_overlapping_operands():
    """out may be the residual (in-place update) but never x or the weight: the epilogue's stores
    would race with other CTAs' loads of them. Checked before any device work, so CPU tensors
    reach the check."""
    from evocompile_b200 import ops

    buf = torch.zeros(64, 64, dtype=torch.bfloat16)
    x, w = buf[:32], torch.zeros(32, 64, dtype=torch.bfloat16)
    resid = torch.zeros(32, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="overlaps x"):
        ops.linear_residual(x, w, resid, out=buf[16:48, :32])
    with pytest.raises(RuntimeError, match="overlaps weight"):
        ops.linear_residual(x, w, resid, out=w[:, :32])
    # disjoint rows of the same buffer and the residual itself pass the check (then the CPU check refuses)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.linear_residual(x, w, resid, out=buf[32:, :32])
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.linear_residual(x, w, resid, out=resid)
