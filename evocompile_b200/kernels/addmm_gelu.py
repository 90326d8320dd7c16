"""gko::addmm_gelu — GEMM + bias + exact-erf GELU on tcgen05 tensor cores.

Drop-in for the reference module eval/kernels/addmm_gelu.py:

* ``torch.ops.gko.addmm_gelu(bias, mat1, mat2)`` (schema of :197-201) computes
  ``gelu(mat1 @ mat2 + bias, approximate="none")`` with mat1 [..., K],
  mat2 [K, N] (usually the W^T view of a Linear weight, read in place) and
  returns a fresh tensor of shape mat1.shape[:-1] + (N,) in mat1's dtype
  (fake at :203-210). bf16/fp16 run the fused tcgen05 kernel; fp32 runs the
  exact-fp32 kernel. Unsupported inputs raise; nothing falls back.
* autograd recomputes the pre-activation and uses gelu_backward, as the
  reference's _addmm_gelu_backward (:175-185).
* ``torch.ops.gko.addmm_gelu_aux(bias, mat1, mat2) -> (out, z)`` and
  ``addmm_gelu_train(bias, mat1, mat2)`` (training form, no reference counterpart):
  the forward kernel also writes the pre-activation z, so the backward runs
  gelu_backward on it and the two gradient GEMMs without recomputing the forward
  GEMM (the recompute the reference notes costs its training steps).
* ``fuse_addmm_gelu(graph)`` rewrites gelu(addmm / F.linear / nn.Linear /
  mm + bias), with up to two view/reshape nodes in between, and the decomposed
  0.5 * x * (1 + erf(x / sqrt 2)) form, into the op (the patterns of :355-512).
* ``register()`` installs the op and the pre-grad + post-grad passes (:527-537).
"""

from __future__ import annotations

from typing import Tuple

import torch

from .. import _lib, ops
from . import gemm_ops

aten = torch.ops.aten

_OP_READY = False
_AUTOGRADED = False
_PASS_INSTALLED = False

_INV_SQRT2 = 0.7071067811865476


def _addmm_gelu_forward(bias, mat1, mat2):
    return ops.addmm_act(bias, mat1, mat2, _lib.ACT_GELU)


def _pre_activation(bias, mat1, mat2):
    """z = mat1 @ mat2 + bias, recomputed on the library GEMM (the reference recomputes it with
    addmm / matmul, eval/kernels/addmm_gelu.py:175-185)."""
    z = torch.ops.gko.gemm(mat1.reshape(-1, mat1.shape[-1]), mat2) + bias
    return z.reshape(*mat1.shape[:-1], mat2.shape[1])


def _weight_grad(mat1, g2):
    """dW = mat1^T @ dZ over all token rows, on the library GEMM with mat1^T read in place."""
    return torch.ops.gko.gemm(mat1.reshape(-1, mat1.shape[-1]).t(), g2)


def _input_grad(g2, mat2, shape):
    """dX = dZ @ mat2^T (mat2^T is the row-major weight of a Linear) on the library GEMM."""
    return torch.ops.gko.gemm(g2, mat2.t()).reshape(shape)


def _setup_context(ctx, inputs, output):
    bias, mat1, mat2 = inputs
    ctx.save_for_backward(bias, mat1, mat2)


def _backward(ctx, grad_output):
    bias, mat1, mat2 = ctx.saved_tensors
    z = _pre_activation(bias, mat1, mat2)
    gz = aten.gelu_backward.default(grad_output, z, approximate="none")
    needs = getattr(ctx, "needs_input_grad", None) or (True, True, True)
    g2 = gz.reshape(-1, gz.shape[-1])
    g_bias = g2.sum(0).reshape(bias.shape) if needs[0] else None
    g_mat1 = _input_grad(g2, mat2, mat1.shape) if needs[1] else None
    g_mat2 = _weight_grad(mat1, g2) if needs[2] else None
    return g_bias, g_mat1, g_mat2


def _setup_aux(ctx, inputs, output):
    bias, mat1, mat2 = inputs
    ctx.save_for_backward(bias, mat1, mat2, output[1])


def _backward_aux(ctx, grad_output, grad_z):
    bias, mat1, mat2, z = ctx.saved_tensors
    gz = aten.gelu_backward.default(grad_output, z, approximate="none")
    if grad_z is not None:
        gz = gz + grad_z
    needs = getattr(ctx, "needs_input_grad", None) or (True, True, True)
    g2 = gz.reshape(-1, gz.shape[-1])
    g_bias = g2.sum(0).reshape(bias.shape) if needs[0] else None
    g_mat1 = _input_grad(g2, mat2, mat1.shape) if needs[1] else None
    g_mat2 = _weight_grad(mat1, g2) if needs[2] else None
    return g_bias, g_mat1, g_mat2


def addmm_gelu_train(bias, mat1, mat2):
    """gelu(mat1 @ mat2 + bias) whose backward reuses the pre-activation saved by the forward kernel."""
    _ensure_op()
    return torch.ops.gko.addmm_gelu_aux(bias, mat1, mat2)[0]


def _ensure_op():
    global _OP_READY, _AUTOGRADED
    gemm_ops.ensure()
    if not _OP_READY:
        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "addmm_gelu")):

            @torch.library.custom_op("gko::addmm_gelu", mutates_args=())
            def addmm_gelu(bias: torch.Tensor, mat1: torch.Tensor, mat2: torch.Tensor) -> torch.Tensor:
                return _addmm_gelu_forward(bias, mat1, mat2)

            @addmm_gelu.register_fake
            def _(bias, mat1, mat2):
                return mat1.new_empty(tuple(mat1.shape[:-1]) + (mat2.shape[-1],))

        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "addmm_gelu_aux")):

            @torch.library.custom_op("gko::addmm_gelu_aux", mutates_args=())
            def addmm_gelu_aux(bias: torch.Tensor, mat1: torch.Tensor,
                               mat2: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
                return ops.addmm_act(bias, mat1, mat2, _lib.ACT_GELU, save_pre=True)

            @addmm_gelu_aux.register_fake
            def _(bias, mat1, mat2):
                shape = (*mat1.shape[:-1], mat2.shape[-1])
                return mat1.new_empty(shape), mat1.new_empty(shape)

            torch.library.register_autograd("gko::addmm_gelu_aux", _backward_aux, setup_context=_setup_aux)

        _OP_READY = True
    if not _AUTOGRADED:
        try:
            torch.library.register_autograd("gko::addmm_gelu", _backward, setup_context=_setup_context)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise
        _AUTOGRADED = True


# --------------------------------------------------------------------------- FX matching
def _target_name(node) -> str:
    return getattr(getattr(node, "target", None), "__name__", "") or ""


def _is_call(node) -> bool:
    return getattr(node, "op", None) in ("call_function", "call_method")


def _module_of(node):
    if getattr(node, "op", None) != "call_module":
        return None
    owner = getattr(node.graph, "owning_module", None)
    if owner is None:
        return None
    try:
        return owner.get_submodule(str(node.target))
    except Exception:
        return None


def _is_exact_gelu(node) -> bool:
    mod = _module_of(node)
    if mod is not None:
        return isinstance(mod, torch.nn.GELU) and getattr(mod, "approximate", "none") in (None, "none")
    if not _is_call(node):
        return False
    tgt = node.target
    if tgt in (aten.gelu.default, aten.gelu, torch.nn.functional.gelu):
        pass
    elif not (_target_name(node) == "gelu" and str(getattr(tgt, "__module__", "")).startswith("torch")):
        return False
    return (node.kwargs or {}).get("approximate", "none") in (None, "none")


def _is_fn(node, *targets, name=None) -> bool:
    if not _is_call(node):
        return False
    if node.target in targets:
        return True
    return name is not None and _target_name(node) == name and not isinstance(node.target, str)


def _is_linear_fn(node) -> bool:
    if not _is_call(node):
        return False
    tgt = node.target
    if tgt in (aten.linear.default, aten.linear, torch.nn.functional.linear, getattr(torch._C._nn, "linear", None)):
        return True
    mod = str(getattr(tgt, "__module__", "") or "")
    return _target_name(node) == "linear" and ("torch" in mod or "aten" in mod)


def _is_view(node) -> bool:
    views = {aten.view.default, aten.reshape.default}
    unsafe = getattr(getattr(aten, "_unsafe_view", None), "default", None)
    if unsafe is not None:
        views.add(unsafe)
    return _is_call(node) and node.target in views


def _const(x):
    return float(x) if isinstance(x, (int, float)) and not isinstance(x, bool) else None


def _scalar_partner(node, operand):
    if not node.args or len(node.args) < 2:
        return None
    a, b = node.args[0], node.args[1]
    if a is operand:
        return _const(b)
    if b is operand:
        return _const(a)
    return None


def _user_scaling(x, factor):
    """The mul(x, factor) user of x, if any."""
    for u in x.users:
        if _is_fn(u, aten.mul.Tensor, aten.mul.default, aten.mul) and _scalar_partner(u, x) is not None:
            if abs(_scalar_partner(u, x) - factor) < 1e-6:
                return u
    return None


def _decomposed_gelu_of(x):
    """Match 0.5 * x * (1 + erf(x * 1/sqrt(2))) hanging off x; returns (output node, nodes)."""
    half = _user_scaling(x, 0.5)
    scaled = _user_scaling(x, _INV_SQRT2)
    if half is None or scaled is None:
        return None
    erfs = [u for u in scaled.users if _is_fn(u, aten.erf.default, aten.erf)]
    if len(erfs) != 1:
        return None
    one_plus = None
    for u in erfs[0].users:
        if _is_fn(u, aten.add.Tensor, aten.add.default, aten.add) and _scalar_partner(u, erfs[0]) == 1.0:
            one_plus = u
    if one_plus is None:
        return None
    for u in one_plus.users:
        if _is_fn(u, aten.mul.Tensor, aten.mul.default, aten.mul) and half in u.args[:2]:
            return u, [u, one_plus, erfs[0], scaled, half]
    return None


class _Site:
    """A GEMM (+ bias) node feeding an exact GELU, with everything the rewrite needs."""

    def __init__(self, gemm, bias, mat1, mat2, weight_rows_n, module_path, extra):
        self.gemm = gemm              # node whose value is the pre-activation
        self.bias = bias
        self.mat1 = mat1
        self.mat2 = mat2              # [K, N] operand, or [N, K] weight when weight_rows_n
        self.weight_rows_n = weight_rows_n
        self.module_path = module_path
        self.extra = extra            # nodes besides `gemm` that become dead


def _gemm_site(src):
    if _is_fn(src, aten.addmm.default, aten.addmm, torch.addmm, name="addmm"):
        b, m1, m2 = src.args[0], src.args[1], src.args[2]
        return _Site(src, b, m1, m2, False, None, [])
    if _is_linear_fn(src):
        args, kw = src.args or (), src.kwargs or {}
        x = args[0] if args else kw.get("input")
        w = args[1] if len(args) > 1 else kw.get("weight")
        b = args[2] if len(args) > 2 else kw.get("bias")
        if x is None or w is None or b is None:
            return None
        return _Site(src, b, x, w, True, None, [])
    mod = _module_of(src)
    if isinstance(mod, torch.nn.Linear) and mod.bias is not None:
        return _Site(src, None, src.args[0], None, True, str(src.target), [])
    if _is_fn(src, aten.add.Tensor, aten.add.default, aten.add) and len(src.args) >= 2:
        for mm, other in ((src.args[0], src.args[1]), (src.args[1], src.args[0])):
            if hasattr(mm, "op") and _is_fn(mm, aten.mm.default, aten.mm) and len(mm.users) == 1:
                s = _Site(src, other, mm.args[0], mm.args[1], False, None, [mm])
                return s
    return None


def _peel_views(node, limit=2):
    views = []
    while hasattr(node, "op") and _is_view(node) and len(views) < limit and node.args:
        views.append(node)
        node = node.args[0]
    return node, views


def fuse_addmm_gelu(graph: torch.fx.Graph) -> int:
    """Rewrite exact-GELU(GEMM + bias) sites of ``graph`` into gko::addmm_gelu. Returns the count."""
    _ensure_op()
    op = torch.ops.gko.addmm_gelu.default
    count = 0
    for node in list(graph.nodes):
        if node.graph is not graph:  # erased earlier in this sweep
            continue
        gelu_out, chain, site, views = None, [], None, []
        if _is_exact_gelu(node):
            src = node.args[0] if node.args else None
            if src is None or not hasattr(src, "op"):
                continue
            src, views = _peel_views(src)
            site = _gemm_site(src)
            gelu_out, chain = node, [node]
        elif _is_fn(node, aten.addmm.default, aten.addmm, torch.addmm, name="addmm"):
            hit = _decomposed_gelu_of(node)
            if hit is None:
                view_users = [u for u in node.users if _is_view(u)]
                if len(view_users) == 1:
                    hit = _decomposed_gelu_of(view_users[0])
                    views = view_users if hit else []
            if hit is None:
                continue
            site = _gemm_site(node)
            gelu_out, chain = hit
        if site is None or gelu_out is None:
            continue
        consumed = set(chain) | set(views)
        if any(u not in consumed for u in site.gemm.users):
            continue  # the pre-activation is needed elsewhere
        if any(u not in consumed for v in views for u in v.users):
            continue
        with graph.inserting_before(gelu_out):
            if site.module_path is not None:
                w = graph.get_attr(site.module_path + ".weight")
                b = graph.get_attr(site.module_path + ".bias")
                mat2 = graph.call_function(aten.t.default, args=(w,))
            else:
                b = site.bias
                mat2 = graph.call_function(aten.t.default, args=(site.mat2,)) if site.weight_rows_n else site.mat2
            new = graph.call_function(op, args=(b, site.mat1, mat2))
            for v in reversed(views):
                new = graph.call_function(v.target, args=(new,) + tuple(v.args[1:]), kwargs=dict(v.kwargs or {}))
        new.meta = dict(gelu_out.meta)
        gelu_out.replace_all_uses_with(new)
        for dead in list(chain) + list(views) + [site.gemm] + site.extra:
            if dead.op != "placeholder" and not dead.users and dead.graph is graph:
                try:
                    graph.erase_node(dead)
                except Exception:
                    pass
        count += 1
    if count:
        graph.lint()
    return count


def _addmm_gelu_pass(graph_or_module) -> None:
    fuse_addmm_gelu(getattr(graph_or_module, "graph", graph_or_module))


_addmm_gelu_pass._gko_graph_native = True  # type: ignore[attr-defined]


def register(backend: str = "") -> None:
    """Install the custom op and the pre-grad (training) and post-grad (inference) passes.

    ``backend`` is accepted for interface compatibility and ignored: there is one backend.
    """
    global _PASS_INSTALLED
    _ensure_op()
    if _PASS_INSTALLED:
        return
    from .pass_install import install_inductor_pass, install_post_grad_pass

    install_inductor_pass("pre_grad_custom_pass", _addmm_gelu_pass, key="addmm_gelu")
    install_post_grad_pass(_addmm_gelu_pass, key="addmm_gelu")
    _PASS_INSTALLED = True
