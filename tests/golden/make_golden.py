"""Generate golden input/output fixtures by running the reference's own Python
operators (EvoCompile eval/kernels, imported from a checkout of the reference)
on the CPU, where they take their eager paths:

  addmm_gelu   torch.ops.gko.addmm_gelu -> _eager_addmm_gelu   (eval/kernels/addmm_gelu.py:81-84)
  gemm_swiglu  gemm_swiglu.apply       -> _eager_gemm_swiglu  (eval/kernels/gemm_swiglu.py:105-109)
  silu_mul     torch.ops.gko.silu_mul  -> _eager              (eval/kernels/silu_mul.py:29-30)
  attention    fused_sdpa.fused_attention -> _fallback (F.sdpa + masks)      (eval/kernels/fused_sdpa.py:508-532)
               cutlass_sdpa.cutlass_attention (window bias, softcap)        (eval/kernels/cutlass_sdpa.py:35-136)
  attention    torch.ops.gko.fused_sdpa with its registered autograd: on the CPU the
  backward    _backward recomputes through _fallback and autograd (eval/kernels/fused_sdpa.py:873-898)

Inputs are drawn from seeded generators and rounded to bfloat16 (stored as
bf16) so the GPU kernels can consume them exactly; outputs are the reference's
fp32 results. Run from the repository root:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [/path/to/EvoCompile]

Writes tests/golden/golden.pt. The reference CPU paths produce no lse, so the
fixtures pin outputs only.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _bf(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(ref_root) / "eval"))
    import kernels  # the reference catalog
    from kernels import cutlass_sdpa, fused_sdpa, gemm_swiglu

    kernels.register("addmm_gelu")
    kernels.register("silu_mul")
    kernels.register("gemm_swiglu")
    torch.backends.cuda.matmul.allow_tf32 = False
    cases = {}

    g = torch.Generator().manual_seed(1234)
    # --- addmm_gelu: 2-D, 3-D (Linear on [B, S, K]) and the fp32 config layout at small size
    for name, xs, n in (("addmm_gelu_2d", (48, 64), 80), ("addmm_gelu_3d", (2, 9, 32), 24), ("addmm_gelu_f32", (32, 128), 256)):
        x = _bf(g, *xs)
        w = _bf(g, n, xs[-1], std=xs[-1] ** -0.5)
        b = _bf(g, n, std=0.02)
        out = torch.ops.gko.addmm_gelu(b.float(), x.float(), w.float().t())
        cases[name] = {"inputs": {"bias": b, "mat1": x, "weight": w}, "out": out.float()}

    # --- gemm_swiglu
    for name, xs, h in (("gemm_swiglu_2d", (40, 64), 48), ("gemm_swiglu_3d", (3, 7, 32), 40)):
        x = _bf(g, *xs)
        w = _bf(g, 2 * h, xs[-1], std=xs[-1] ** -0.5)
        out = gemm_swiglu.apply(x.float(), w.float())
        cases[name] = {"inputs": {"x": x, "weight": w}, "out": out.float()}

    # --- silu_mul
    x, y = _bf(g, 3, 50), _bf(g, 3, 50)
    cases["silu_mul"] = {"inputs": {"x": x, "y": y}, "out": torch.ops.gko.silu_mul(x.float(), y.float()).float()}

    # --- attention through the reference's CPU paths
    def qkv(z, h, s, d):
        return _bf(g, z, h, s, d), _bf(g, z, h, s, d), _bf(g, z, h, s, d)

    for causal in (0, 1):
        q, k, v = qkv(2, 2, 40, 64)
        out = fused_sdpa.fused_attention(q.float(), k.float(), v.float(), None, 0.125, causal)
        cases[f"attn_plain_c{causal}"] = {"inputs": {"q": q, "k": k, "v": v}, "out": out.float(),
                                          "args": {"scale": 0.125, "causal": causal}}
    q, k, v = qkv(2, 2, 33, 64)
    pad = torch.zeros(2, 33)
    pad[1, -5:] = torch.finfo(torch.float32).min
    out = fused_sdpa.fused_attention(q.float(), k.float(), v.float(), pad, 0.125, 0)
    cases["attn_keypad"] = {"inputs": {"q": q, "k": k, "v": v, "bias": pad}, "out": out.float(),
                            "args": {"scale": 0.125, "causal": 0}}
    q, k, v = qkv(2, 2, 24, 64)
    rel = (torch.randn(1, 2, 24, 24, generator=g) * 0.5)
    out = fused_sdpa.fused_attention(q.float(), k.float(), v.float(), rel, 0.125, 1)
    cases["attn_relbias_causal"] = {"inputs": {"q": q, "k": k, "v": v, "bias": rel}, "out": out.float(),
                                    "args": {"scale": 0.125, "causal": 1}}
    q, k, v = qkv(1, 2, 48, 64)
    out = cutlass_sdpa.cutlass_attention(q.float(), k.float(), v.float(), None, 0.125, 1, 8, 0.0)
    cases["attn_window_causal"] = {"inputs": {"q": q, "k": k, "v": v}, "out": out.float(),
                                   "args": {"scale": 0.125, "causal": 1, "window": 8}}
    q, k, v = qkv(1, 2, 32, 64)
    out = cutlass_sdpa.cutlass_attention(q.float(), k.float(), v.float(), None, 0.5, 0, 0, 5.0)
    cases["attn_softcap"] = {"inputs": {"q": q, "k": k, "v": v}, "out": out.float(),
                             "args": {"scale": 0.5, "causal": 0, "softcap": 5.0}}

    # --- attention backward: dq, dk, dv of <out, dO> through the reference's catalog op
    fused_sdpa._ensure_op()
    for causal, bias_kind in ((0, None), (1, None), (0, "keypad")):
        q, k, v = qkv(2, 2, 40, 64)
        do = _bf(g, 2, 2, 40, 64)
        bias = torch.empty(0)
        if bias_kind == "keypad":
            bias = torch.zeros(2, 40)
            bias[0, -7:] = torch.finfo(torch.float32).min
        qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
        out = torch.ops.gko.fused_sdpa(qf, kf, vf, bias, 0.125, causal)
        dq, dk, dv = torch.autograd.grad(out, (qf, kf, vf), do.float())
        name = f"attn_bwd_c{causal}" + (f"_{bias_kind}" if bias_kind else "")
        cases[name] = {"inputs": {"q": q, "k": k, "v": v, "dout": do, "bias": bias},
                       "out": out.detach().float(), "dq": dq.float(), "dk": dk.float(), "dv": dv.float(),
                       "args": {"scale": 0.125, "causal": causal}}

    meta = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
            "reference": "EvoCompile eval/kernels (CPU eager paths)"}
    torch.save({"meta": meta, "cases": cases}, HERE / "golden.pt")
    print(f"wrote {HERE / 'golden.pt'} with {len(cases)} cases")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EVOCOMPILE_REF")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py <EvoCompile checkout root> "
                 "(or set EVOCOMPILE_REF); the root holds eval/kernels")
    main(root)
