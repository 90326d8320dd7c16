"""Install FX graph passes into Inductor's custom-pass slots.

Same interface as the reference's eval/kernels/pass_install.py (install_inductor_pass
:70-90, install_post_grad_pass :92-93, normalize_pre_pass :96-102, reset_passes
:105-114, install_generated_pass :117-136), so catalog modules and generated
kernels register their rewrites the same way. Each slot holds one callable that
runs every installed pass in order; installation is idempotent per (slot, key).
A pass may be written against a Graph or a GraphModule; Inductor hands either.
"""

from __future__ import annotations

from typing import Any, Callable, Iterable

_SLOTS = ("pre_grad_custom_pass", "post_grad_custom_pre_pass")
_installed: dict[str, list[tuple[str, Callable]]] = {}
_keys: set[str] = set()


class _GraphModuleView:
    """Lets a pass written for a GraphModule run on a bare Graph."""

    def __init__(self, graph: Any) -> None:
        self.graph = graph

    def recompile(self) -> None:
        self.graph.lint()


def as_graph_pass(fn: Callable) -> Callable:
    """Wrap ``fn`` so that it accepts a Graph or a GraphModule."""
    if getattr(fn, "_gko_graph_wrapped", False) or getattr(fn, "_gko_graph_native", False):
        return fn
    if hasattr(fn, "uuid"):  # an Inductor CustomGraphPass object
        return fn

    def run(graph_or_module: Any) -> Any:
        is_module = hasattr(graph_or_module, "graph") and callable(getattr(graph_or_module, "recompile", None))
        return fn(graph_or_module if is_module else _GraphModuleView(graph_or_module))

    run.__name__ = getattr(fn, "__name__", "gko_pass")
    run._gko_graph_wrapped = True  # type: ignore[attr-defined]
    return run


def _chain(fns: Iterable[Callable]) -> Callable:
    fns = [f for f in fns if f is not None]

    def run(graph: Any) -> None:
        for f in fns:
            f(graph)

    run.__name__ = "gko_chained_pass"
    run._gko_graph_native = True  # type: ignore[attr-defined]
    return run


def ensure_graph_pass(fn: Any) -> Any:
    """Normalise a pass, or a list of passes, into one callable."""
    if fn is None:
        return None
    if isinstance(fn, (list, tuple)):
        return _chain(ensure_graph_pass(f) for f in fn)
    return as_graph_pass(fn)


def install_inductor_pass(attr: str, pass_fn: Callable, *, key: str = "") -> None:
    """Append ``pass_fn`` to Inductor config slot ``attr`` unless ``key`` is already there."""
    import torch._inductor.config as cfg

    if not callable(pass_fn):
        raise TypeError(f"install_inductor_pass({attr!r}, ...): pass_fn must be callable, got {type(pass_fn).__name__}")
    if not hasattr(cfg, attr):
        return
    token = f"{attr}:{key or getattr(pass_fn, '__name__', '') or id(pass_fn)}"
    if token in _keys:
        return
    wrapped = ensure_graph_pass(pass_fn)
    current = getattr(cfg, attr)
    setattr(cfg, attr, wrapped if current is None else _chain([current, wrapped]))
    _keys.add(token)


def install_post_grad_pass(pass_fn: Callable, *, key: str = "") -> None:
    install_inductor_pass("post_grad_custom_pre_pass", pass_fn, key=key)


def normalize_pre_pass() -> None:
    """Make whatever sits in the post-grad slot callable on a Graph."""
    import torch._inductor.config as cfg

    cur = cfg.post_grad_custom_pre_pass
    if cur is not None:
        cfg.post_grad_custom_pre_pass = ensure_graph_pass(cur)


def reset_passes() -> None:
    """Forget every installed pass (the next evaluation sees only its own recipe)."""
    _keys.clear()
    try:
        import torch._inductor.config as cfg
    except Exception:
        return
    for slot in _SLOTS:
        if hasattr(cfg, slot):
            setattr(cfg, slot, None)


def install_generated_pass(mod: Any, name: str) -> None:
    """Install the FX pass of a generated kernel module whose register() could not."""
    fn = getattr(mod, "_post_grad_pass", None)
    if fn is None:
        for attr in sorted(dir(mod)):
            if attr in ("_PASS_INSTALLED", "register") or not attr.startswith("_"):
                continue
            obj = getattr(mod, attr, None)
            low = attr.lower()
            if callable(obj) and (low.endswith("_pass") or "rewrite" in low or "fx_pass" in low or low.endswith("_pattern")):
                fn = obj
                break
    if fn is None:
        raise AttributeError(f"generated kernel {name} has no post-grad pass to install")
    install_inductor_pass("pre_grad_custom_pass", fn, key=name)
    install_post_grad_pass(fn, key=name)
