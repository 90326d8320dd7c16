"""ctypes binding of libgko_b200.so (the C ABI declared in include/gko_b200.h).

The library is the product path: there is no fallback. If it is missing or a
CUDA device is absent, every operator raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libgko_b200.so"

F16, BF16, F32 = 1, 2, 3
ACT_NONE, ACT_GELU, ACT_RELU = 0, 1, 2
BIAS_NONE, BIAS_KEYPAD, BIAS_FULL = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3

_DTYPE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

_lib = None
_lock = threading.Lock()

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_fl = ctypes.c_float
_p64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); every symbol of include/gko_b200.h
SIGNATURES = {
    "gko_last_error": (ctypes.c_char_p, []),
    "gko_version": (_int, []),
    "gko_addmm_act": (
        _int,
        [_int, _int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _int, _vp, _i64, _vp, _vp],
    ),
    "gko_linear_swiglu": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp],
    ),
    "gko_fmha_fwd": (
        _int,
        [_int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _int, _int,
         _p64, _i64, _p64, _fl, _int, _int, _fl, _vp, _vp, _vp, _vp],
    ),
    "gko_fmha_varlen_fwd": (
        _int,
        [_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _i64, _vp, _vp, _fl, _int, _int, _fl, _vp, _vp, _vp, _vp],
    ),
    "gko_fmha_bwd_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _int]),
    "gko_fmha_bwd": (
        _int,
        [_int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _int, _int,
         _p64, _i64, _vp, _p64, _vp, _p64, _vp, _fl, _int, _int, _fl, _vp, _p64, _vp, _p64, _vp, _p64,
         _vp, _i64, _vp, _vp],
    ),
    "gko_fmha_bwd_noalloc": (
        _int,
        [_int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _int, _int,
         _p64, _i64, _vp, _p64, _vp, _p64, _vp, _fl, _int, _int, _fl, _vp, _p64, _vp, _p64, _vp, _p64,
         _vp, _vp],
    ),
    "gko_fmha_varlen_bwd": (
        _int,
        [_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _fl, _int, _int, _fl, _vp, _i64, _i64, _vp,
         _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp],
    ),
    "gko_linear_allreduce": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _int, _vp, _vp],
    ),
    "gko_addmm_act_aux": (
        _int,
        [_int, _int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _int, _vp, _i64, _vp, _i64, _vp, _vp],
    ),
    "gko_linear_swiglu_aux": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp],
    ),
    "gko_linear_residual": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp],
    ),
    "gko_rms_stats": (_int, [_int, _i64, _i64, _vp, _vp, _fl, _vp, _vp, _i64, _vp, _vp]),
    "gko_linear_rowscale": (
        _int,
        [_int, _int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp],
    ),
    "gko_linear_rowscale_rope": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _fl, _vp, _vp],
    ),
    "gko_set_gemm_ctas": (_int, [_int]),
    "gko_allreduce_residual_nvls": (_int, [_int, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _fl, _vp, _vp]),
    "gko_swiglu_bwd": (_int, [_int, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp]),
    "gko_silu_mul": (_int, [_int, _i64, _vp, _vp, _vp, _vp, _vp]),
    "gko_selftest_wait_timeout": (_int, [_vp, ctypes.c_longlong, _vp]),
    "gko_rmsnorm": (_int, [_int, _i64, _i64, _vp, _vp, _vp, _fl, _vp, _vp, _i64, _vp, _vp]),
    "gko_rope": (_int, [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _fl, _vp, _vp]),
}


def load():
    """Load libgko_b200.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m evocompile_b200.build` "
                "(the fused operators have no fallback implementation)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().gko_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != OK:
        kind = {ERR_INVALID: "invalid argument", ERR_UNSUPPORTED: "unsupported input",
                ERR_CUDA: "CUDA error"}.get(rc, f"error {rc}")
        raise RuntimeError(f"{what}: {kind}: {last_error()}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE[t]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t}; the fused operators take float16, bfloat16 or float32")


_status = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels OR their timeout bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = w
    return w


def read_status(device: torch.device, clear: bool = True) -> int:
    """Synchronise and return the device status word (0 = no kernel timed out)."""
    w = status_word(device)
    v = int(w.item())
    if clear and v:
        w.zero_()
    return v


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "gko fused operators run only on CUDA tensors (sm_100a); got a tensor on "
                f"{t.device} — there is no CPU fallback"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"operands on different devices: {dev} and {t.device}")
    load()
    return dev
