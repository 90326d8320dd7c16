"""gko_fmha_bwd_noalloc: the attention backward for callers that cannot allocate
device memory (their memory is held by another runtime's pool, they cannot afford
cudaMalloc's synchronisation, or they are plain C code with no allocator). It takes
its workspace from a fixed 32 MiB array inside the library instead of an argument.

Called here through the C ABI on two problems in a row (the second reuses the array
the first left behind) and compared with gko_fmha_bwd, which gets a fresh workspace;
also checks that a problem too large for the array is refused with a clear error.
This file is collected last so that a run stopping at its first failure has already
run every other test.
"""

import ctypes

import pytest
import torch

import oracle
from evocompile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 3e-2  # the tolerance of the attention backward tests
_I64x4 = ctypes.c_int64 * 4


def _vp(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _noalloc(q, k, v, out, lse, dout, scale, causal, d=None):
    z, hq, sq, d_ = q.shape
    d = d_ if d is None else d
    hkv, sk = k.shape[1], k.shape[2]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dev = q.device
    rc = _lib.load().gko_fmha_bwd_noalloc(
        _lib.dtype_code(q.dtype), z, hq, hkv, sq, sk, d,
        _vp(q), _I64x4(*q.stride()), _vp(k), _I64x4(*k.stride()), _vp(v), _I64x4(*v.stride()),
        _vp(None), _lib.BIAS_NONE, 0, _I64x4(0, 0, 0, 0), 1,
        _vp(out), _I64x4(*out.stride()), _vp(dout), _I64x4(*dout.stride()), _vp(lse),
        float(scale), int(causal), 0, 0.0,
        _vp(dq), _I64x4(*dq.stride()), _vp(dk), _I64x4(*dk.stride()), _vp(dv), _I64x4(*dv.stride()),
        ctypes.c_void_p(_lib.status_word(dev).data_ptr()), ctypes.c_void_p(_lib.stream_ptr(dev)),
    )
    _lib.check(rc, "gko_fmha_bwd_noalloc")
    return dq, dk, dv


def _problem(seed, z, hq, hkv, s, d, causal):
    g = torch.Generator().manual_seed(seed)
    mk = lambda h: torch.randn(z, h, s, d, generator=g).to(torch.bfloat16).cuda()  # noqa: E731
    q, k, v, dout = mk(hq), mk(hkv), mk(hkv), mk(hq)
    out, lse = ops.fmha_fwd(q, k, v, None, d ** -0.5, causal)
    return q, k, v, out, lse, dout


@pytest.mark.parametrize("case", [(0, 2, 8, 2, 1000, 128, 1), (1, 3, 4, 4, 333, 64, 0)])
def test_noalloc_matches_workspace_entry_point_twice(case):
    seed, z, hq, hkv, s, d, causal = case
    for call in range(2):  # the second call starts from the scratch the first one left
        q, k, v, out, lse, dout = _problem(seed * 10 + call, z, hq, hkv, s + 37 * call, d, causal)
        ref = ops.fmha_bwd(q, k, v, None, out, lse, dout, d ** -0.5, causal)
        got = _noalloc(q, k, v, out, lse, dout, d ** -0.5, causal)
        torch.cuda.synchronize()
        assert _lib.read_status(q.device) == 0
        for g, r in zip(got, ref):
            assert torch.isfinite(g.float()).all()
            assert oracle.rel_err(g, r) <= TOL


def test_noalloc_rejects_problems_beyond_the_scratch():
    z, hq, hkv, s, d = 1, 16, 16, 4160, 128  # 16 * 65 = 1040 blocks > 1008
    t = torch.zeros(z, hq, s, d, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(z * hq, s, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="scratch"):
        _noalloc(t, t, t, t, lse, t, 0.1, 1)


def test_noalloc_argument_errors_match_workspace_entry_point():
    """A head dim the kernels do not implement is refused with the same error as gko_fmha_bwd
    (the head-dim rule), before the scratch size is computed."""
    t = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(2, 64, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="head dim 64 or 128"):
        _noalloc(t, t, t, t, lse, t, 0.1, 1, d=96)
