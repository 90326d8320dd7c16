"""Tensor-parallel decomposition of the Llama block on CPU with two gloo ranks: each rank
computes its shard (column-parallel QKV / gate-up, row-parallel o / down) in fp32 and the
all-reduced result equals the unsharded block. This covers the host-side partitioning that the
GPU path (evocompile_b200.block.TPBlock) uses with NCCL."""

import os
import random

import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

import oracle
from evocompile_b200.block import BlockConfig, init_weights, shard_weights

CFG = BlockConfig(d_model=128, n_heads=8, n_kv_heads=4, head_dim=32, d_ff=256)


def _tp_forward(local, cfg, x, group):
    """The TPBlock.forward data flow with fp32 CPU ops and a gloo all-reduce."""
    B, S, d = x.shape
    hd, hq, hkv = cfg.head_dim, local["hq_local"], local["hkv_local"]
    h = oracle.rmsnorm(x, local["attn_norm"], cfg.eps)
    qkv = F.linear(h, local["wqkv"].float())
    q = qkv[..., : hq * hd].reshape(B, S, hq, hd)
    k = qkv[..., hq * hd: (hq + hkv) * hd].reshape(B, S, hkv, hd)
    v = qkv[..., (hq + hkv) * hd:].reshape(B, S, hkv, hd)
    q = torch.stack([oracle.rope(q[b], cfg.rope_theta) for b in range(B)])
    k = torch.stack([oracle.rope(k[b], cfg.rope_theta) for b in range(B)])
    o, _ = oracle.attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, hd ** -0.5, 1)
    o = F.linear(o.transpose(1, 2).reshape(B, S, hq * hd), local["wo"].float())
    dist.all_reduce(o, group=group)
    x1 = x + o
    h2 = oracle.rmsnorm(x1, local["mlp_norm"], cfg.eps)
    gu = F.linear(h2, local["w_gate_up"].float())
    g = F.silu(gu[..., : gu.shape[-1] // 2]) * gu[..., gu.shape[-1] // 2:]
    dn = F.linear(g, local["w_down"].float())
    dist.all_reduce(dn, group=group)
    return x1 + dn


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = init_weights(CFG, "cpu", torch.float32, seed=0)
        x = torch.randn(2, 24, CFG.d_model, generator=torch.Generator().manual_seed(1))
        y = _tp_forward(shard_weights(full, CFG, rank, world), CFG, x, None)
        if rank == 0:
            ref = oracle.llama_block(x, full, CFG)
            q.put(float((y - ref).abs().max() / ref.abs().max()))
    finally:
        dist.destroy_process_group()


def test_shard_shapes():
    full = init_weights(CFG, "cpu", torch.float32)
    for world in (1, 2, 4):
        loc = shard_weights(full, CFG, 0, world)
        hd = CFG.head_dim
        assert loc["wqkv"].shape == ((CFG.n_heads + 2 * CFG.n_kv_heads) // world * hd, CFG.d_model)
        assert loc["wo"].shape == (CFG.d_model, CFG.n_heads // world * hd)
        assert loc["w_gate_up"].shape == (2 * CFG.d_ff // world, CFG.d_model)
        assert loc["w_down"].shape == (CFG.d_model, CFG.d_ff // world)


def test_flops_formula():
    cfg = BlockConfig()
    assert abs(cfg.flops(16384, 4096) - 2.914e13) / 2.914e13 < 2e-3


def test_tp2_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + random.Random().randint(0, 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-5


def test_comm_auto_policy(monkeypatch):
    """comm="auto" sums row-parallel outputs inside the GEMM on two ranks, with NCCL on four and
    through the NVLS row-slice reduction on eight (the fastest form measured at each); explicit
    modes are kept; others are rejected."""
    from evocompile_b200.block import TPBlock

    local = shard_weights(init_weights(CFG, torch.device("cpu"), torch.float32, seed=1), CFG, 0, 1)
    for world, want in ((2, "fused"), (4, "nccl"), (8, "nvls")):
        monkeypatch.setattr(dist, "get_world_size", lambda group=None, w=world: w)
        assert TPBlock(local, CFG, group=object()).comm == want
        assert TPBlock(local, CFG, group=object(), comm="fused").comm == "fused"
        assert TPBlock(local, CFG, group=object(), comm="nvls_pipe").comm == "nvls_pipe"
    import pytest

    with pytest.raises(ValueError):
        TPBlock(local, CFG, comm="ring")


def test_post_attention_schedule_orders_each_stream():
    """Every step appears once; on each stream the steps of a chunk follow its dependencies
    (o before its all-reduce, that all-reduce before the chunk's MLP, the MLP before the down
    all-reduce), so the two in-order streams cannot wait on each other in a cycle."""
    from evocompile_b200.block import post_attention_schedule

    for chunks in (1, 2, 4, 7):
        order = post_attention_schedule(chunks)
        assert sorted(order) == sorted((k, c) for c in range(chunks) for k in ("o", "ar_o", "mlp", "ar_d"))
        pos = {step: i for i, step in enumerate(order)}
        for c in range(chunks):
            assert pos[("o", c)] < pos[("ar_o", c)] < pos[("mlp", c)] < pos[("ar_d", c)]
        compute = [s for s in order if s[0] in ("o", "mlp")]
        comm = [s for s in order if s[0] in ("ar_o", "ar_d")]
        # a step waits only on steps of the other stream issued before it in the global order:
        # simulate both in-order streams to completion
        done, ic, im = set(), 0, 0
        deps = {("ar_o", c): ("o", c) for c in range(chunks)}
        deps.update({("mlp", c): ("ar_o", c) for c in range(chunks)})
        deps.update({("ar_d", c): ("mlp", c) for c in range(chunks)})
        while ic < len(compute) or im < len(comm):
            moved = False
            if ic < len(compute) and deps.get(compute[ic], None) in (None, *done):
                done.add(compute[ic]); ic += 1; moved = True
            if im < len(comm) and deps[comm[im]] in done:
                done.add(comm[im]); im += 1; moved = True
            assert moved, f"streams deadlock at {compute[ic:ic + 1]} / {comm[im:im + 1]}"
    import pytest

    with pytest.raises(ValueError):
        post_attention_schedule(0)


def _chunked_worker(rank, world, port, q):
    """The pipelined data flow (per-chunk all-reduces of the o-projection and down outputs) on CPU
    ranks equals the unsharded block."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from evocompile_b200.block import post_attention_schedule
        from evocompile_b200.shard import row_range

        full = init_weights(CFG, "cpu", torch.float32, seed=0)
        local = shard_weights(full, CFG, rank, world)
        x = torch.randn(1, 30, CFG.d_model, generator=torch.Generator().manual_seed(1))
        B, S, d = x.shape
        hd, hq, hkv = CFG.head_dim, local["hq_local"], local["hkv_local"]
        h = oracle.rmsnorm(x, local["attn_norm"], CFG.eps)
        qkv = F.linear(h, local["wqkv"].float())
        qh = oracle.rope(qkv[0, :, : hq * hd].reshape(S, hq, hd), CFG.rope_theta)
        kh = oracle.rope(qkv[0, :, hq * hd: (hq + hkv) * hd].reshape(S, hkv, hd), CFG.rope_theta)
        vh = qkv[0, :, (hq + hkv) * hd:].reshape(S, hkv, hd)
        att, _ = oracle.attention(qh.transpose(0, 1)[None], kh.transpose(0, 1)[None], vh.transpose(0, 1)[None],
                                  None, hd ** -0.5, 1)
        attn2d = att[0].transpose(0, 1).reshape(S, hq * hd)
        x2 = x[0]
        chunks = 4
        rng = [row_range(S, c, chunks) for c in range(chunks)]
        y = torch.empty(S, d)
        o = {}
        for kind, c in post_attention_schedule(chunks):
            a, b = rng[c]
            if kind == "o":
                o[c] = F.linear(attn2d[a:b], local["wo"].float())
            elif kind == "ar_o":
                dist.all_reduce(o[c])
            elif kind == "mlp":
                x1 = x2[a:b] + o[c]
                h2 = oracle.rmsnorm(x1, local["mlp_norm"], CFG.eps)
                gu = F.linear(h2, local["w_gate_up"].float())
                g = F.silu(gu[:, : gu.shape[-1] // 2]) * gu[:, gu.shape[-1] // 2:]
                y[a:b] = F.linear(g, local["w_down"].float()) + (x1 if rank == 0 else 0)
            else:
                dist.all_reduce(y[a:b])
        if rank == 0:
            ref = oracle.llama_block(x, full, CFG)[0]
            q.put(float((y - ref).abs().max() / ref.abs().max()))
    finally:
        dist.destroy_process_group()


def test_pipelined_tp2_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 32600 + random.Random().randint(0, 2000)
    procs = [ctx.Process(target=_chunked_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-5


def test_nvls_chunk_slices_partition_rows():
    """The pipelined NVSwitch form reduces, per token chunk [a, b), the slice
    a + row_range(b - a, rank, world) on each rank: over all chunks and ranks every row of the
    block's output is summed exactly once (ragged chunk and rank splits included)."""
    from evocompile_b200.shard import row_range

    for T in (1, 7, 320, 16384, 16387):
        for chunks in (1, 3, 4, 7):
            for world in (2, 4, 8):
                seen = [0] * T
                for c in range(max(1, min(chunks, T))):
                    a, b = row_range(T, c, max(1, min(chunks, T)))
                    for r in range(world):
                        r0, r1 = row_range(b - a, r, world)
                        assert a <= a + r0 <= a + r1 <= b
                        for i in range(a + r0, a + r1):
                            seen[i] += 1
                assert seen == [1] * T, (T, chunks, world)
