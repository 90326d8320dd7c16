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
