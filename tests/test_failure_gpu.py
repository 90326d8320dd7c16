"""Failure detection on the GPU without a fault: a wait that can never complete
ends after its time limit with a status bit, and the context stays usable."""

import ctypes

import pytest
import torch

from evocompile_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _lib.load().gko_selftest_wait_timeout(ctypes.c_void_p(status.data_ptr()), 50_000_000,
                                               ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc, "selftest")
    torch.cuda.synchronize(dev)
    assert int(status.item()) & 0x1, "the stalled wait did not report a timeout"
    # the context still runs kernels correctly afterwards
    x = torch.randn(128, 64, device=dev).to(torch.bfloat16)
    w = torch.randn(128, 64, device=dev).to(torch.bfloat16)
    out = ops.addmm_act(None, x, w.t(), _lib.ACT_NONE)
    ref = x.float() @ w.float().t()
    assert (out.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


def test_host_rejects_bad_selftest_args():
    with pytest.raises(RuntimeError, match="limit"):
        _lib.check(_lib.load().gko_selftest_wait_timeout(ctypes.c_void_p(8), -1, ctypes.c_void_p(0)), "selftest")
