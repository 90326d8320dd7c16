"""gko::silu_mul — silu(x) * y in one HBM-bound CUDA kernel, plus its FX pass.

Drop-in for eval/kernels/silu_mul.py: op schema (:71-73), fake (:75-77),
autograd (:51-58), the mul(silu(a), b) rewrite (:103-128) and register() (:139-148).
"""

from __future__ import annotations

import torch

from .. import ops

aten = torch.ops.aten

_OP_READY = False
_AUTOGRADED = False
_PASS_INSTALLED = False


def _setup_context(ctx, inputs, output):
    x, y = inputs
    ctx.save_for_backward(x, y)


def _backward(ctx, grad_out):
    x, y = ctx.saved_tensors
    sig = torch.sigmoid(x)
    return grad_out * y * (sig * (1 + x * (1 - sig))), grad_out * (x * sig)


def _ensure_op():
    global _OP_READY, _AUTOGRADED
    if not _OP_READY:
        if not (hasattr(torch.ops, "gko") and hasattr(torch.ops.gko, "silu_mul")):

            @torch.library.custom_op("gko::silu_mul", mutates_args=())
            def silu_mul(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
                return ops.silu_mul(x, y)

            @silu_mul.register_fake
            def _(x, y):
                return torch.empty_like(x, memory_format=torch.contiguous_format)

        _OP_READY = True
    if not _AUTOGRADED:
        try:
            torch.library.register_autograd("gko::silu_mul", _backward, setup_context=_setup_context)
        except RuntimeError as e:
            if "already" not in str(e).lower():
                raise
        _AUTOGRADED = True


def _is_silu(node) -> bool:
    tgt = getattr(node, "target", None)
    return tgt in (aten.silu.default, aten.silu, torch.nn.functional.silu) or getattr(tgt, "__name__", "") == "silu"


def _is_mul(node) -> bool:
    return getattr(node, "target", None) in (aten.mul.Tensor, aten.mul.default, aten.mul)


def fuse_silu_mul(graph) -> int:
    """Rewrite mul(silu(a), b) (either operand order, silu used once) into gko::silu_mul."""
    _ensure_op()
    op = torch.ops.gko.silu_mul.default
    n = 0
    for node in list(graph.nodes):
        if not _is_mul(node) or len(node.args) < 2:
            continue
        a, b = node.args[0], node.args[1]
        if hasattr(a, "op") and _is_silu(a) and len(a.users) == 1:
            silu_node, other = a, b
        elif hasattr(b, "op") and _is_silu(b) and len(b.users) == 1:
            silu_node, other = b, a
        else:
            continue
        if not hasattr(other, "op"):
            continue  # a python scalar operand is not an elementwise tensor product
        with graph.inserting_before(node):
            new = graph.call_function(op, args=(silu_node.args[0], other))
        new.meta = dict(node.meta)
        node.replace_all_uses_with(new)
        graph.erase_node(node)
        if not silu_node.users:
            graph.erase_node(silu_node)
        n += 1
    if n:
        graph.lint()
    return n


def _pass(graph_or_module) -> None:
    fuse_silu_mul(getattr(graph_or_module, "graph", graph_or_module))


_pass._gko_graph_native = True  # type: ignore[attr-defined]


def register(backend: str = "") -> None:
    global _PASS_INSTALLED
    _ensure_op()
    if _PASS_INSTALLED:
        return
    from .pass_install import install_inductor_pass, install_post_grad_pass

    install_inductor_pass("pre_grad_custom_pass", _pass, key="silu_mul")
    install_post_grad_pass(_pass, key="silu_mul")
    _PASS_INSTALLED = True
