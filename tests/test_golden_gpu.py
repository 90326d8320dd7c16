"""The CUDA kernels against the reference-generated golden vectors
(tests/golden/golden.pt) — bf16 inputs, fp32 reference outputs.
Tolerance: max|err| / max|ref| <= 2e-2 (bf16/fp16 outputs), 1e-3 for fp32 outputs."""

from pathlib import Path

import pytest
import torch

import oracle
from evocompile_b200 import ops

pytestmark = pytest.mark.gpu

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=False)["cases"]


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("addmm_gelu")])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_addmm_gelu_golden(name, dtype):
    c = GOLDEN[name]
    i = {k: v.cuda().to(dtype) for k, v in c["inputs"].items()}
    out = ops.addmm_act(i["bias"], i["mat1"], i["weight"].t())
    assert oracle.rel_err(out, c["out"]) <= (1e-3 if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("gemm_swiglu")])
def test_gemm_swiglu_golden(name):
    c = GOLDEN[name]
    out = ops.linear_swiglu(c["inputs"]["x"].cuda(), c["inputs"]["weight"].cuda())
    assert oracle.rel_err(out, c["out"]) <= 2e-2


def test_silu_mul_golden():
    c = GOLDEN["silu_mul"]
    out = ops.silu_mul(c["inputs"]["x"].cuda(), c["inputs"]["y"].cuda())
    assert oracle.rel_err(out, c["out"]) <= 2e-2


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("attn_")])
def test_attention_golden(name):
    c = GOLDEN[name]
    i, a = c["inputs"], c["args"]
    bias = i.get("bias")
    out, _ = ops.fmha_fwd(i["q"].cuda(), i["k"].cuda(), i["v"].cuda(), None if bias is None else bias.cuda(),
                          a["scale"], a["causal"], a.get("window", 0), a.get("softcap", 0.0))
    assert oracle.rel_err(out, c["out"]) <= 2e-2


@pytest.mark.parametrize("name", [n for n in GOLDEN if n.startswith("attn_bwd")])
def test_attention_bwd_golden(name):
    """The tcgen05 backward (forward out / lse from the library) against the reference's dq, dk, dv."""
    c = GOLDEN[name]
    i, a = c["inputs"], c["args"]
    q, k, v, do = (i[n].cuda() for n in ("q", "k", "v", "dout"))
    bias = i["bias"].cuda() if i["bias"].numel() else None
    out, lse = ops.fmha_fwd(q, k, v, bias, a["scale"], a["causal"])
    dq, dk, dv = ops.fmha_bwd(q, k, v, bias, out, lse, do, a["scale"], a["causal"])
    for got, ref in ((dq, c["dq"]), (dk, c["dk"]), (dv, c["dv"])):
        assert oracle.rel_err(got, ref) <= 3e-2
