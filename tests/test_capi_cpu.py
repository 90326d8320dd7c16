"""The C ABI on a machine without a GPU: libgko_b200.so loads, exports every
function include/gko_b200.h declares, and rejects bad arguments before any
CUDA call with the documented error codes and messages."""

import ctypes
import re
from pathlib import Path

from evocompile_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "gko_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gko_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("gko_addmm_act", "gko_linear_swiglu", "gko_fmha_fwd", "gko_fmha_varlen_fwd", "gko_silu_mul",
              "gko_last_error", "gko_version"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in gko_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version(lib):
    assert lib.gko_version() >= 100


def _null():
    return ctypes.c_void_p(0)


def test_addmm_rejects_unknown_dtype(lib):
    rc = lib.gko_addmm_act(99, 1, 4, 4, 4, _null(), 4, 1, _null(), 1, 4, _null(), 0, _null(), 4, _null(), _null())
    assert rc == _lib.ERR_INVALID
    assert "dtype" in _lib.last_error()


def test_addmm_rejects_unknown_activation(lib):
    rc = lib.gko_addmm_act(_lib.BF16, 7, 4, 4, 4, _null(), 4, 1, _null(), 1, 4, _null(), 0, _null(), 4, _null(), _null())
    assert rc == _lib.ERR_INVALID and "activation" in _lib.last_error()


def test_addmm_rejects_negative_and_null(lib):
    assert lib.gko_addmm_act(_lib.BF16, 1, -1, 4, 4, _null(), 4, 1, _null(), 1, 4, _null(), 0, _null(), 4,
                             _null(), _null()) == _lib.ERR_INVALID
    assert lib.gko_addmm_act(_lib.BF16, 1, 4, 4, 4, _null(), 4, 1, _null(), 1, 4, _null(), 0, _null(), 4,
                             _null(), _null()) == _lib.ERR_INVALID
    assert "null" in _lib.last_error()


def test_empty_gemm_is_a_no_op(lib):
    assert lib.gko_addmm_act(_lib.BF16, 1, 0, 4, 4, _null(), 4, 1, _null(), 1, 4, _null(), 0, _null(), 4,
                             _null(), _null()) == _lib.OK


def test_tensor_core_layout_constraints(lib):
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    # K % 8 != 0 -> unsupported (stride rule of the TMA descriptors)
    rc = lib.gko_addmm_act(_lib.BF16, 1, 16, 16, 12, fake, 12, 1, fake, 1, 12, _null(), 0, fake, 16, _null(), _null())
    assert rc == _lib.ERR_UNSUPPORTED and "multiples of 8" in _lib.last_error()
    # transposed mat1 with an activation: the MN-major A path has the plain epilogue only
    rc = lib.gko_addmm_act(_lib.BF16, 1, 16, 16, 16, fake, 1, 16, fake, 1, 16, _null(), 0, fake, 16, _null(), _null())
    assert rc == _lib.ERR_UNSUPPORTED and "without an activation" in _lib.last_error()
    # mat1 with no unit stride at all
    rc = lib.gko_addmm_act(_lib.BF16, 0, 16, 16, 16, fake, 32, 2, fake, 1, 16, _null(), 0, fake, 16, _null(), _null())
    assert rc == _lib.ERR_UNSUPPORTED and "unit stride in one dimension" in _lib.last_error()


def _i64x4(*v):
    return (ctypes.c_int64 * 4)(*v)


def test_fmha_rejects_head_dim_and_dtype(lib):
    st = _i64x4(0, 0, 0, 1)
    args = lambda dt, d, hq=4, hkv=2: (dt, 1, hq, hkv, 16, 16, d, _null(), st, _null(), st, _null(), st, _null(), 0, 0,
                                      st, 1, None, 0.1, 0, 0, 0.0, _null(), _null(), _null(), _null())
    assert lib.gko_fmha_fwd(*args(_lib.BF16, 96)) == _lib.ERR_UNSUPPORTED
    assert "head dim" in _lib.last_error()
    assert lib.gko_fmha_fwd(*args(_lib.F32, 64)) == _lib.ERR_UNSUPPORTED
    assert lib.gko_fmha_fwd(*args(_lib.BF16, 64, 4, 3)) == _lib.ERR_INVALID
    assert "multiple of kv heads" in _lib.last_error()


def test_fmha_varlen_rejects_negative(lib):
    rc = lib.gko_fmha_varlen_fwd(_lib.BF16, -1, 4, 4, 128, 10, 10, 10, _null(), 512, 128, _null(), 512, 128,
                                 _null(), 512, 128, _null(), _null(), 0.1, 1, 0, 0.0, _null(), _null(), _null(), _null())
    assert rc == _lib.ERR_INVALID


def test_silu_mul_validation(lib):
    assert lib.gko_silu_mul(_lib.BF16, -3, _null(), _null(), _null(), _null(), _null()) == _lib.ERR_INVALID
    assert lib.gko_silu_mul(_lib.BF16, 0, _null(), _null(), _null(), _null(), _null()) == _lib.OK
    assert lib.gko_silu_mul(_lib.BF16, 8, _null(), _null(), _null(), _null(), _null()) == _lib.ERR_INVALID


def test_allreduce_residual_nvls_validation(lib):
    """The NVSwitch row-slice reduction refuses bad arguments on the host, before any launch; an
    empty row range is a no-op."""
    def call(dtype=_lib.BF16, rows=64, cols=512, ld=512, r0=0, r1=32, part=16, res=0, out=16, inv=0):
        return lib.gko_allreduce_residual_nvls(dtype, rows, cols, ld, r0, r1, ctypes.c_void_p(part),
                                               ctypes.c_void_p(res), ctypes.c_void_p(out), ctypes.c_void_p(inv),
                                               1e-5, _null(), _null())

    assert call(dtype=_lib.F32) == _lib.ERR_UNSUPPORTED and "bf16 or f16" in _lib.last_error()
    assert call(r1=65) == _lib.ERR_INVALID and "bad sizes" in _lib.last_error()
    assert call(r0=10, r1=5) == _lib.ERR_INVALID
    assert call(ld=256) == _lib.ERR_INVALID
    assert call(cols=100, ld=104) == _lib.ERR_UNSUPPORTED and "cols % 8" in _lib.last_error()
    assert call(cols=16392, ld=16392) == _lib.ERR_UNSUPPORTED
    assert call(r0=7, r1=7) == _lib.OK  # nothing to reduce: no launch, no CUDA call
    assert call(part=0) == _lib.ERR_INVALID and "multicast" in _lib.last_error()
    assert call(part=8) == _lib.ERR_UNSUPPORTED and "16-byte" in _lib.last_error()
    assert call(inv=18) == _lib.ERR_UNSUPPORTED


def test_gemm_cta_cap_setter(lib):
    """gko_set_gemm_ctas returns the previous cap (0 = every SM) and refuses negative values."""
    prev = lib.gko_set_gemm_ctas(5)
    try:
        assert prev == 0
        assert lib.gko_set_gemm_ctas(9) == 5
        assert lib.gko_set_gemm_ctas(-1) == -1 and ">= 0" in _lib.last_error()
        assert lib.gko_set_gemm_ctas(9) == 9
    finally:
        lib.gko_set_gemm_ctas(prev)
