"""Attention backend policy — a single backend.

The reference picks Triton or CUTLASS per model kind (eval/kernels/attn_policy.py:29-64).
This library has exactly one attention kernel, so the policy keeps the same
functions for callers (the attention rewrite calls ``set_context``) and always
resolves to it.
"""

from __future__ import annotations

import os

BACKEND = "b200"
_N_LAYER = 0
_KIND = ""


def resolve(kind, n_layer):
    return BACKEND


def set_context(n_layer=0, kind=""):
    global _N_LAYER, _KIND
    _N_LAYER, _KIND = int(n_layer or 0), str(kind or "")
    os.environ["GKO_ATTN_N_LAYER"] = str(_N_LAYER)
    os.environ["GKO_ATTN_KIND"] = _KIND
    os.environ["GKO_ATTN_RESOLVED"] = BACKEND


def resolved():
    return BACKEND
