"""Tensor-parallel row-parallel linear with the all-reduce inside the GEMM.

``FusedAllReduceLinear`` owns an output buffer in symmetric memory (every rank's copy
mapped into every other rank's address space over NVLink, plus an NVLink multicast address
when the switch supports it). A call computes this rank's partial x @ W^T with the tcgen05
GEMM whose epilogue adds each finished output chunk into all ranks' copies — one in-switch
reduction per 16 bytes through the multicast address (NVLS), or one reduction per peer
without it — so the sum over the group is complete in every rank's buffer when the kernel
ends; no separate all-reduce pass reads the partials back from HBM.

Sequence on the current stream: zero this rank's copy, group barrier (every copy is zero
before any rank adds), fused GEMM + reduction, group barrier (every rank's additions have
landed before any rank reads). The returned tensor is the buffer itself: it is valid until
the next call on the same object, which the stream order already guarantees for consumers
on the same stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, ops


class FusedAllReduceLinear:
    def __init__(self, rows: int, cols: int, dtype, device, group, use_multicast: bool = True):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.world = dist.get_world_size(group)
        self.buf = symm_mem.empty((rows, cols), dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        mc = int(self.handle.multicast_ptr or 0)
        self.multicast = mc if (use_multicast and mc) else 0
        self.peers = int(self.handle.buffer_ptrs_dev)

    def __call__(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """x [rows, k] (this rank's input slice) @ weight [cols, k]^T, summed over the group."""
        if tuple(x.shape[:-1]) != (self.buf.shape[0],) or weight.shape[0] != self.buf.shape[1]:
            raise RuntimeError(f"FusedAllReduceLinear built for [{self.buf.shape[0]}, {self.buf.shape[1]}] output, "
                               f"got x {tuple(x.shape)} weight {tuple(weight.shape)}")
        self.buf.zero_()
        self.handle.barrier(channel=0)
        ops.linear_allreduce(x, weight, self.buf, self.multicast, self.peers, self.world)
        self.handle.barrier(channel=0)
        return self.buf


def p2p_reduction_check(rows: int = 16384, cols: int = 8192, k: int = 14336, iters: int = 5, seed: int = 0) -> dict:
    """One process driving two GPUs: the row-parallel GEMM on cuda:0 adds its partial x @ W^T into
    an output on cuda:0 and one on cuda:1 through the epilogue's peer reductions (the path the
    fused all-reduce takes without a multicast address), against a torch fp32 reference. A
    diagnostic of this machine's NVLink peer path, and a single-process target for a profiler.

    Peer access between the two devices is enabled explicitly (cudaDeviceEnablePeerAccess) and
    the check refuses to run without it: a reduction into a peer address the device may not reach
    would fault. Returns the relative error on each device and the mean device time per GEMM."""
    from cuda.bindings import runtime as rt

    if torch.cuda.device_count() < 2:
        raise RuntimeError("p2p_reduction_check needs two GPUs")
    for dev, peer in ((0, 1), (1, 0)):
        ok, can = rt.cudaDeviceCanAccessPeer(dev, peer)
        if ok != rt.cudaError_t.cudaSuccess or not can:
            raise RuntimeError(f"cuda:{dev} cannot access cuda:{peer} as a peer")
        (e,) = rt.cudaSetDevice(dev)
        if e != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaSetDevice({dev}): {e}")
        torch.cuda.set_device(dev)
        torch.empty(1, device=f"cuda:{dev}")  # the device's primary context exists before enabling
        (e,) = rt.cudaDeviceEnablePeerAccess(peer, 0)
        if e not in (rt.cudaError_t.cudaSuccess, rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
            raise RuntimeError(f"cudaDeviceEnablePeerAccess({dev} -> {peer}): {e}")
    torch.cuda.set_device(0)
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    g = torch.Generator(device=d0).manual_seed(seed)
    x = torch.randn(rows, k, device=d0, generator=g).to(torch.bfloat16)
    w = (torch.randn(cols, k, device=d0, generator=g) * k ** -0.5).to(torch.bfloat16)
    out0 = torch.empty(rows, cols, device=d0, dtype=torch.bfloat16)
    out1 = torch.empty(rows, cols, device=d1, dtype=torch.bfloat16)
    peers = torch.tensor([out0.data_ptr(), out1.data_ptr()], dtype=torch.int64, device=d0)
    ms = []
    for _ in range(iters):
        out0.zero_()
        out1.zero_()
        torch.cuda.synchronize(d1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.linear_allreduce(x, w, out0, 0, peers.data_ptr(), 2)
        b.record()
        torch.cuda.synchronize(d0)
        ms.append(a.elapsed_time(b))
    torch.cuda.synchronize(d1)
    status = _lib.read_status(d0)
    ref = x.float() @ w.float().t()
    err = lambda o: ((o.float().to(d0) - ref).abs().max() / ref.abs().max()).item()  # noqa: E731
    return {"rel_err_cuda0": err(out0), "rel_err_cuda1": err(out1), "ms_per_gemm": sum(ms[1:]) / max(1, len(ms) - 1),
            "status": status, "rows": rows, "cols": cols, "k": k,
            "nvlink_bytes_algorithmic": rows * cols * 2}


if __name__ == "__main__":
    import argparse
    import json

    ap = argparse.ArgumentParser(description="two-GPU check of the GEMM epilogue's peer reductions")
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=8192)
    ap.add_argument("--k", type=int, default=14336)
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args()
    print(json.dumps(p2p_reduction_check(a.rows, a.cols, a.k, a.iters)))


class NvlsResidualReduce:
    """The sum over the group of a row-parallel projection's output, plus a residual (and the
    RMSNorm statistics of the result), through NVLink multicast (``gko_allreduce_residual_nvls``).

    A call: the GEMM writes this rank's partial into its copy of a symmetric buffer (no
    communication), group barrier, every rank sums its slice of the rows over all ranks in the
    switch, adds the residual and writes the rows (and 1/rms per row) to every rank's copy of the
    output buffers, group barrier. Returns (out, inv) — the symmetric output buffer and the fp32
    statistics (None without ``stats``), valid until the next call on this object.
    """

    def __init__(self, rows: int, cols: int, dtype, device, group, stats: bool):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.partial = symm_mem.empty((rows, cols), dtype=dtype, device=device)
        self.hp = symm_mem.rendezvous(self.partial, group.group_name)
        self.out = symm_mem.empty((rows, cols), dtype=dtype, device=device)
        self.ho = symm_mem.rendezvous(self.out, group.group_name)
        self.inv = self.hi = None
        if stats:
            self.inv = symm_mem.empty((rows,), dtype=torch.float32, device=device)
            self.hi = symm_mem.rendezvous(self.inv, group.group_name)
        for h in (self.hp, self.ho, self.hi):
            if h is not None and not int(h.multicast_ptr or 0):
                raise RuntimeError("NvlsResidualReduce needs NVLink multicast (NVLS) on this group")

    def __call__(self, x: torch.Tensor, weight: torch.Tensor, resid, eps: float = 1e-5):
        rows, cols = self.partial.shape
        if tuple(x.shape[:-1]) != (rows,) or weight.shape[0] != cols:
            raise RuntimeError(f"NvlsResidualReduce built for [{rows}, {cols}], got x {tuple(x.shape)} "
                               f"weight {tuple(weight.shape)}")
        ops.linear(x, weight, out=self.partial)
        self.reduce_rows(0, rows, resid, eps)
        return self.out, self.inv

    def reduce_rows(self, a: int, b: int, resid, eps: float = 1e-5) -> None:
        """Sum rows [a, b) of the partials over the group, on the current stream: barrier (every
        rank has written those rows of its partial), this rank's slice of [a, b) reduced in the
        switch (plus the residual's rows, and the statistics) and stored to every rank's copy of
        the output, barrier (every rank's stores have landed). Rows outside [a, b) are untouched,
        so consecutive row ranges can be reduced while later rows' partials are still being
        computed on another stream. ``resid``: the whole contiguous [rows, cols] residual, or None."""
        from .shard import row_range

        rows, cols = self.partial.shape
        if not 0 <= a <= b <= rows:
            raise RuntimeError(f"NvlsResidualReduce: rows [{a}, {b}) outside [0, {rows})")
        dev = self.partial.device
        if resid is not None and (tuple(resid.shape) != (rows, cols) or resid.stride() != (cols, 1)
                                  or resid.dtype != self.partial.dtype or resid.device != dev):
            raise RuntimeError("NvlsResidualReduce: the residual is a contiguous [rows, cols] tensor of the "
                               "output's dtype on the same device")
        r0, r1 = row_range(b - a, self.rank, self.world)
        self.hp.barrier(channel=0)
        with torch.cuda.device(dev):
            rc = _lib.load().gko_allreduce_residual_nvls(
                _lib.dtype_code(self.partial.dtype), rows, cols, cols, a + r0, a + r1,
                ctypes.c_void_p(int(self.hp.multicast_ptr)),
                ctypes.c_void_p(resid.data_ptr() if resid is not None else 0),
                ctypes.c_void_p(int(self.ho.multicast_ptr)),
                ctypes.c_void_p(int(self.hi.multicast_ptr) if self.hi is not None else 0), float(eps),
                ctypes.c_void_p(_lib.status_word(dev).data_ptr()), ctypes.c_void_p(_lib.stream_ptr(dev)))
        _lib.check(rc, "gko_allreduce_residual_nvls")
        self.hp.barrier(channel=0)
