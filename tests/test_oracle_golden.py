"""Pin the CPU oracle against golden vectors produced by the reference's own
operators (tests/golden/make_golden.py): the oracle must reproduce the
reference's fp32 outputs to fp32 rounding."""

from pathlib import Path

import pytest
import torch

import oracle

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=False)["cases"]


def _close(a, b, tol=1e-5):
    assert a.shape == b.shape
    assert oracle.rel_err(a, b) <= tol, oracle.rel_err(a, b)


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("addmm_gelu")])
def test_addmm_gelu_golden(name):
    c = GOLDEN[name]
    i = c["inputs"]
    _close(oracle.addmm_gelu(i["bias"], i["mat1"], i["weight"].t()), c["out"])


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("gemm_swiglu")])
def test_gemm_swiglu_golden(name):
    c = GOLDEN[name]
    _close(oracle.gemm_swiglu(c["inputs"]["x"], c["inputs"]["weight"]), c["out"])


def test_silu_mul_golden():
    c = GOLDEN["silu_mul"]
    _close(oracle.silu_mul(c["inputs"]["x"], c["inputs"]["y"]), c["out"])


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("attn_")])
def test_attention_golden(name):
    c = GOLDEN[name]
    i, a = c["inputs"], c["args"]
    out, _ = oracle.attention(i["q"], i["k"], i["v"], i.get("bias"), a["scale"], a["causal"],
                              a.get("window", 0), a.get("softcap", 0.0))
    _close(out, c["out"], 2e-5)


def test_oracle_gqa_matches_sdpa_enable_gqa():
    """GQA has no reference path; cross-check the oracle's head grouping against
    torch's own scaled_dot_product_attention(enable_gqa=True)."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 8, 30, 64, generator=g)
    k = torch.randn(2, 2, 30, 64, generator=g)
    v = torch.randn(2, 2, 30, 64, generator=g)
    out, _ = oracle.attention(q, k, v, None, 0.125, 1)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=0.125, is_causal=True, enable_gqa=True)
    _close(out, ref, 2e-5)


def test_oracle_varlen_is_per_sequence_dense():
    g = torch.Generator().manual_seed(1)
    lens = [5, 17, 1]
    cu = torch.tensor([0, 5, 22, 23], dtype=torch.int32)
    q = torch.randn(23, 4, 64, generator=g)
    k = torch.randn(23, 2, 64, generator=g)
    v = torch.randn(23, 2, 64, generator=g)
    out, lse = oracle.attention_varlen(q, k, v, cu, cu, 0.125, 1)
    for i, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        o, l = oracle.attention(q[a:b].transpose(0, 1)[None], k[a:b].transpose(0, 1)[None],
                                v[a:b].transpose(0, 1)[None], None, 0.125, 1)
        _close(out[a:b], o[0].transpose(0, 1), 1e-6)
        assert torch.allclose(lse[:, a:b], l.view(4, b - a))


def test_oracle_lse_matches_logsumexp():
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(1, 2, 16, 64, generator=g) for _ in range(3))
    _, lse = oracle.attention(q, k, v, None, 0.3, 0)
    ref = torch.logsumexp(torch.matmul(q, k.transpose(-1, -2)) * 0.3, dim=-1).reshape(2, 16)
    assert torch.allclose(lse, ref, atol=1e-5)


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("attn_bwd")])
def test_attention_bwd_golden(name):
    """The oracle's backward (autograd of its fp32 restatement) against dq, dk, dv from the
    reference's gko::fused_sdpa autograd on the CPU."""
    c = GOLDEN[name]
    i, a = c["inputs"], c["args"]
    dq, dk, dv = oracle.attention_bwd(i["q"], i["k"], i["v"], i["dout"], i["bias"], a["scale"], a["causal"])
    _close(dq, c["dq"], 2e-5)
    _close(dk, c["dk"], 2e-5)
    _close(dv, c["dv"], 2e-5)


def test_oracle_bwd_matches_finite_differences():
    """dL/dx of L = <attention(q, k, v), dO> by central differences in float64 (GQA, causal, softcap)."""
    g = torch.Generator().manual_seed(7)
    q = torch.randn(1, 4, 9, 16, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 11, 16, generator=g, dtype=torch.float64)
    v = torch.randn(1, 2, 11, 16, generator=g, dtype=torch.float64)
    do = torch.randn(1, 4, 9, 16, generator=g, dtype=torch.float64)
    dq, dk, dv = oracle.attention_bwd(q, k, v, do, None, 0.3, 1, 0, 2.0)

    def loss(q_, k_, v_):
        return float((oracle.attention(q_, k_, v_, None, 0.3, 1, 0, 2.0)[0].double() * do).sum())

    eps = 1e-3
    for t, grad, idx in ((q, dq, (0, 3, 5, 7)), (k, dk, (0, 1, 4, 2)), (v, dv, (0, 0, 2, 9))):
        tp, tm = t.clone(), t.clone()
        tp[idx] += eps
        tm[idx] -= eps
        args_p = [tp if x is t else x for x in (q, k, v)]
        args_m = [tm if x is t else x for x in (q, k, v)]
        fd = (loss(*args_p) - loss(*args_m)) / (2 * eps)
        assert abs(fd - float(grad[idx])) <= 1e-3 * max(1.0, abs(fd)), (fd, float(grad[idx]))
