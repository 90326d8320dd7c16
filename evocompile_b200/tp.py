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
