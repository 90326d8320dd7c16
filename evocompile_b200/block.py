"""Llama-3-70B-shaped transformer block (prefill) on the fused operators, tensor-parallel.

    x -> RMSNorm -> QKV GEMM -> RoPE(q, k) -> causal GQA attention -> o-proj -> all-reduce
      -> + x -> RMSNorm -> gate/up GEMM + SwiGLU -> down GEMM -> all-reduce -> + residual

Megatron-style split over ``world`` ranks (one process per GPU): the QKV projection is
column-parallel by kv group (each rank owns Hkv/world kv heads and the Hq/world query heads
that use them), the o-projection row-parallel; gate/up column-parallel (each rank owns
d_ff/world gate rows and the matching up rows), the down projection row-parallel. The two
row-parallel outputs are summed with an NCCL all-reduce. RMSNorm weights are replicated.

Every GEMM is the tcgen05 kernel (the SwiGLU one fused), attention the tcgen05 FMHA reading
q/k/v in place from the QKV output and writing [tokens, heads, d] for the o-projection.
RoPE runs in the QKV GEMM's epilogue on the fp32 accumulator (head dim 128); the RMSNorm
statistics (``ops.rms_stats``: 1/rms per token, plus the residual sum) are a memory-bound kernel; each RMSNorm is applied as a per-row scale in the epilogue of the
GEMM that follows it, with its weight folded into that GEMM's weight (``ops.linear_rowscale``), so
the normalised activations never go to HBM; the closing residual
add runs in the down projection's epilogue (``ops.linear_residual``) on one rank, and with NCCL
on rank 0 before the all-reduce. With
``comm="fused"`` the two row-parallel projections reduce their outputs across the group
inside the GEMM over NVLink (``evocompile_b200.tp.FusedAllReduceLinear``); ``comm="nccl"``
runs the GEMM and then an NCCL all-reduce. ``comm="auto"`` (the default) picks the fused
form on two ranks, NCCL on four and the NVLS row-slice reduction on eight: with the fused form each
rank's GEMM shrinks with the rank count while its NVLink reduction traffic stays the whole output, so
its reductions stop hiding behind the GEMM's main loop as the rank count grows.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass(frozen=True)
class BlockConfig:
    d_model: int = 8192
    n_heads: int = 64
    n_kv_heads: int = 8
    head_dim: int = 128
    d_ff: int = 28672
    eps: float = 1e-5
    rope_theta: float = 500000.0

    def flops(self, tokens: int, seq_len: int) -> float:
        """Algorithmic FLOP of one block forward over `tokens` tokens in sequences of `seq_len` (causal)."""
        d, hd = self.d_model, self.head_dim
        qkv = 2.0 * tokens * d * (self.n_heads + 2 * self.n_kv_heads) * hd
        attn = 2.0 * self.n_heads * hd * seq_len * seq_len * (tokens / seq_len)  # causal half of 4·H·S²·D per seq
        oproj = 2.0 * tokens * self.n_heads * hd * d
        gateup = 2.0 * tokens * d * 2 * self.d_ff
        down = 2.0 * tokens * self.d_ff * d
        return qkv + attn + oproj + gateup + down


WEIGHT_NAMES = ("attn_norm", "wq", "wk", "wv", "wo", "mlp_norm", "w_gate", "w_up", "w_down")


def init_weights(cfg: BlockConfig, device, dtype=torch.bfloat16, seed: int = 0, std: float = 0.02):
    """Full (unsharded) random-init weights: projections ~ N(0, std), norm weights 1."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, hd = cfg.d_model, cfg.head_dim

    def w(rows, cols):
        return (torch.randn(rows, cols, device=device, generator=g) * std).to(dtype)

    return {
        "attn_norm": torch.ones(d, device=device, dtype=dtype),
        "wq": w(cfg.n_heads * hd, d),
        "wk": w(cfg.n_kv_heads * hd, d),
        "wv": w(cfg.n_kv_heads * hd, d),
        "wo": w(d, cfg.n_heads * hd),
        "mlp_norm": torch.ones(d, device=device, dtype=dtype),
        "w_gate": w(cfg.d_ff, d),
        "w_up": w(cfg.d_ff, d),
        "w_down": w(d, cfg.d_ff),
    }


def shard_weights(full: dict, cfg: BlockConfig, rank: int, world: int) -> dict:
    """This rank's slice of the block weights (column-parallel QKV and gate/up, row-parallel o/down).

    Returns wqkv [(hq_l + 2 hkv_l) * D, d] (rows: local q heads, then local k heads, then local v heads),
    wo [d, hq_l * D], w_gate_up [2 * ff_l, d] (local gate rows then local up rows), w_down [d, ff_l],
    and the replicated norm weights.
    """
    if cfg.n_kv_heads % world or cfg.n_heads % world or cfg.d_ff % world:
        raise ValueError(f"world {world} must divide kv heads {cfg.n_kv_heads}, heads and d_ff")
    hd = cfg.head_dim
    hkv_l = cfg.n_kv_heads // world
    hq_l = cfg.n_heads // world
    ff_l = cfg.d_ff // world
    q_rows = slice(rank * hq_l * hd, (rank + 1) * hq_l * hd)
    kv_rows = slice(rank * hkv_l * hd, (rank + 1) * hkv_l * hd)
    ff = slice(rank * ff_l, (rank + 1) * ff_l)
    return {
        "attn_norm": full["attn_norm"],
        "mlp_norm": full["mlp_norm"],
        "wqkv": torch.cat([full["wq"][q_rows], full["wk"][kv_rows], full["wv"][kv_rows]], 0).contiguous(),
        "wo": full["wo"][:, q_rows].contiguous(),
        "w_gate_up": torch.cat([full["w_gate"][ff], full["w_up"][ff]], 0).contiguous(),
        "w_down": full["w_down"][:, ff].contiguous(),
        "hq_local": hq_l,
        "hkv_local": hkv_l,
    }


def post_attention_schedule(chunks: int) -> list:
    """Issue order of the token-chunk pipeline after attention (every step past attention is
    per token, so the tokens split into ``chunks`` row ranges that flow independently):

    * ("o", c): o-projection GEMM of chunk c (compute stream);
    * ("ar_o", c): all-reduce of its output (communication stream, after ("o", c));
    * ("mlp", c): residual add + RMSNorm statistics, gate/up and down GEMMs of chunk c (compute
      stream, after ("ar_o", c));
    * ("ar_d", c): all-reduce of the down output (communication stream, after ("mlp", c)).

    Each stream runs its steps in list order. The o-projection of chunk c+1 is issued before the
    MLP of chunk c, so the compute stream has work while chunk c's o-projection is being summed,
    and every all-reduce but the last overlaps a later chunk's GEMMs."""
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    order = []
    for c in range(chunks):
        order += [("o", c), ("ar_o", c)]
        if c:
            order += [("mlp", c - 1), ("ar_d", c - 1)]
    order += [("mlp", chunks - 1), ("ar_d", chunks - 1)]
    return order


class TPBlock:
    """One rank of the tensor-parallel block. ``group`` is a torch.distributed process group
    (NCCL) or None for a single GPU.

    ``comm``: "fused" sums the row-parallel outputs inside the GEMM over NVLink; "nccl" runs each
    row-parallel GEMM then a blocking NCCL all-reduce; "nvls" writes each row-parallel partial to
    symmetric memory and sums it in the NVSwitch, each rank reducing a slice of the rows with the
    residual add and the next RMSNorm's statistics folded in (``tp.NvlsResidualReduce``); "pipe" splits the tokens after attention
    into ``chunks`` and pipelines them (``post_attention_schedule``): each chunk's all-reduces run
    on a communication stream while later chunks' GEMMs run, with the GEMMs capped at all SMs but
    ``comm_sms`` so that NCCL's kernels have SMs of their own; "nvls_pipe" is the same token-chunk
    pipeline with each chunk summed by the NVSwitch reduction of "nvls" instead of NCCL; "auto"
    picks per rank count."""

    def __init__(self, local: dict, cfg: BlockConfig, group=None, comm: str = "auto", chunks: int = 4,
                 comm_sms: int = 16):
        if comm not in ("auto", "fused", "nccl", "pipe", "nvls", "nvls_pipe"):
            raise ValueError(f"comm must be 'auto', 'fused', 'nccl', 'pipe', 'nvls' or 'nvls_pipe', got {comm!r}")
        self.chunks = chunks
        self.comm_sms = comm_sms
        self._comm_stream = None
        # RMSNorm runs as a per-row scale in the epilogue of the GEMM that follows it, with the
        # norm weight folded into that GEMM's weight once here: w'[n, j] = w[n, j] * g[j]
        self.w = dict(local)
        self.w["wqkv_n"] = ops.fold_rmsnorm_weight(self.w.pop("wqkv"), local["attn_norm"])
        self.w["w_gate_up_n"] = ops.fold_rmsnorm_weight(self.w.pop("w_gate_up"), local["mlp_norm"])
        self.cfg = cfg
        self.group = group
        self.world = 1 if group is None else torch.distributed.get_world_size(group)
        if comm == "auto":
            # measured on B200 for the B=4 S=4096 block: TP2 in-GEMM 11.82 ms vs NCCL 12.19; TP4 NCCL
            # 6.67 vs NVLS 6.76 vs in-GEMM 7.33; TP8 NVLS 4.07 vs NCCL 4.47 vs in-GEMM 8.54
            comm = "fused" if self.world == 2 else ("nvls" if self.world >= 8 else "nccl")
        self.comm = comm
        self._fused = {}

    def _row_parallel(self, x, weight, slot, resid=None, mark=None):
        """x @ weight^T summed over the group (row-parallel projection), plus ``resid`` (replicated
        on every rank, updated in place) when given. ``mark(name)``, if given, is called between
        the GEMM and the NCCL all-reduce (the fused form has no such boundary)."""
        if self.world == 1:
            if resid is not None:
                return ops.linear_residual(x, weight, resid, out=resid)
            return ops.linear(x, weight)
        if self.comm == "nccl":
            # rank 0 adds the residual in its GEMM epilogue, so the all-reduce sums it in once
            if resid is not None and torch.distributed.get_rank(self.group) == 0:
                y = ops.linear_residual(x, weight, resid, out=resid)
            else:
                y = ops.linear(x, weight)
            if mark is not None:
                mark(f"{('o_proj', 'down')[slot]}_gemm")
            torch.distributed.all_reduce(y, op=torch.distributed.ReduceOp.SUM, group=self.group)
            return y
        from .tp import FusedAllReduceLinear

        key = (slot, x.shape[0], weight.shape[0], x.dtype)
        f = self._fused.get(key)
        if f is None:  # collective: every rank builds it at the same call
            f = FusedAllReduceLinear(x.shape[0], weight.shape[0], x.dtype, x.device, self.group)
            self._fused[key] = f
        y = f(x, weight)
        return y if resid is None else resid.add_(y)

    def _nvls(self, slot, rows, cols, dtype, device, stats):
        from .tp import NvlsResidualReduce

        key = ("nvls", slot, rows, cols, dtype)
        r = self._fused.get(key)
        if r is None:  # collective: every rank builds it at the same call
            r = NvlsResidualReduce(rows, cols, dtype, device, self.group, stats)
            self._fused[key] = r
        return r

    def _comm(self, device):
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device)
        return self._comm_stream

    def _post_attention_nvls_pipelined(self, attn2d, x2):
        """``_post_attention_pipelined`` with each chunk's sums done by the NVSwitch reductions
        (``tp.NvlsResidualReduce.reduce_rows``): the o-projection and down GEMMs of a chunk write
        its rows of this rank's partial into symmetric memory on the compute stream; on the
        communication stream the chunk's rows are summed in the switch with the residual added
        (and, after the o-projection, the RMSNorm statistics computed) while the next chunks'
        GEMMs run. Returns the block output [T, d]."""
        from .shard import row_range

        w, cfg = self.w, self.cfg
        T, d = x2.shape
        chunks = max(1, min(self.chunks, T))
        rng = [row_range(T, c, chunks) for c in range(chunks)]
        cur = torch.cuda.current_stream()
        comm = self._comm(x2.device)
        r_o = self._nvls(0, T, d, x2.dtype, x2.device, True)
        r_d = self._nvls(1, T, d, x2.dtype, x2.device, False)
        x1, inv2 = r_o.out, r_o.inv  # summed o-projection + residual, and its 1/rms per row
        done_o, done_ar, done_mlp = {}, {}, {}
        comm.wait_stream(cur)
        sms = torch.cuda.get_device_properties(x2.device).multi_processor_count
        prev = ops.set_gemm_ctas(max(1, sms - self.comm_sms))
        try:
            for kind, c in post_attention_schedule(chunks):
                a, b = rng[c]
                if kind == "o":
                    ops.linear(attn2d[a:b], w["wo"], out=r_o.partial[a:b])
                    done_o[c] = torch.cuda.Event()
                    done_o[c].record(cur)
                elif kind == "ar_o":
                    comm.wait_event(done_o[c])
                    with torch.cuda.stream(comm):
                        r_o.reduce_rows(a, b, x2, cfg.eps)
                        done_ar[c] = torch.cuda.Event()
                        done_ar[c].record(comm)
                elif kind == "mlp":
                    cur.wait_event(done_ar[c])
                    g = ops.linear_rowscale(x1[a:b], w["w_gate_up_n"], inv2[a:b], swiglu=True)
                    ops.linear(g, w["w_down"], out=r_d.partial[a:b])
                    done_mlp[c] = torch.cuda.Event()
                    done_mlp[c].record(cur)
                else:  # "ar_d"
                    comm.wait_event(done_mlp[c])
                    with torch.cuda.stream(comm):
                        r_d.reduce_rows(a, b, x1, cfg.eps)
        finally:
            ops.set_gemm_ctas(prev)
        cur.wait_stream(comm)
        return r_d.out.clone()  # the symmetric buffer is rewritten by the next call

    def _post_attention_pipelined(self, attn2d, x2):
        """o-projection, residual, RMSNorm, SwiGLU MLP and both all-reduces, token chunk by token
        chunk (``post_attention_schedule``); returns the block output [T, d]."""
        from .shard import row_range

        w, cfg = self.w, self.cfg
        T, d = x2.shape
        chunks = max(1, min(self.chunks, T))
        rng = [row_range(T, c, chunks) for c in range(chunks)]
        cur = torch.cuda.current_stream()
        comm = self._comm(x2.device)
        rank0 = torch.distributed.get_rank(self.group) == 0
        y = torch.empty(T, d, device=x2.device, dtype=x2.dtype)
        o, x1, done_o, done_ar, done_mlp = {}, {}, {}, {}, {}
        sms = torch.cuda.get_device_properties(x2.device).multi_processor_count
        prev = ops.set_gemm_ctas(max(1, sms - self.comm_sms))
        try:
            for kind, c in post_attention_schedule(chunks):
                a, b = rng[c]
                if kind == "o":
                    o[c] = ops.linear(attn2d[a:b], w["wo"])
                    done_o[c] = torch.cuda.Event()
                    done_o[c].record(cur)
                elif kind == "ar_o":
                    comm.wait_event(done_o[c])
                    with torch.cuda.stream(comm):
                        torch.distributed.all_reduce(o[c], op=torch.distributed.ReduceOp.SUM, group=self.group)
                        done_ar[c] = torch.cuda.Event()
                        done_ar[c].record(comm)
                elif kind == "mlp":
                    cur.wait_event(done_ar[c])
                    inv2, x1[c] = ops.rms_stats(o[c], cfg.eps, residual=x2[a:b])
                    g = ops.linear_rowscale(x1[c], w["w_gate_up_n"], inv2, swiglu=True)
                    if rank0:  # the residual is summed in once, by rank 0's GEMM epilogue
                        ops.linear_residual(g, w["w_down"], x1[c], out=y[a:b])
                    else:
                        ops.linear(g, w["w_down"], out=y[a:b])
                    done_mlp[c] = torch.cuda.Event()
                    done_mlp[c].record(cur)
                else:  # "ar_d"
                    comm.wait_event(done_mlp[c])
                    with torch.cuda.stream(comm):
                        torch.distributed.all_reduce(y[a:b], op=torch.distributed.ReduceOp.SUM, group=self.group)
        finally:
            ops.set_gemm_ctas(prev)
        cur.wait_stream(comm)
        y.record_stream(comm)
        return y

    def forward(self, x: torch.Tensor, events=None, mark=None) -> torch.Tensor:
        """x [B, S, d_model] (bf16) -> [B, S, d_model]. ``events`` (start, end) CUDA events, if
        given, bracket the fused gate/up kernel (for per-kernel timing). ``mark(name)``, if given,
        is called at each phase boundary on the launching stream (``start``, ``qkv``, ``attention``,
        ``o_proj``, ``norm2``, ``gate_up``, ``down``; with NCCL also ``o_proj_gemm`` and
        ``down_gemm`` between each GEMM and its all-reduce), so a caller can record a CUDA event
        per boundary and time each phase."""
        cfg, w = self.cfg, self.w
        B, S, d = x.shape
        T, hd = B * S, cfg.head_dim
        hq, hkv = w["hq_local"], w["hkv_local"]
        mk = mark if mark is not None else (lambda name: None)
        mk("start")
        x2 = x.reshape(T, d)
        inv1 = ops.rms_stats(x2, cfg.eps)                                 # 1/rms per token (fp32)
        # rmsnorm(x) Wqkv^T [T, (hq + 2 hkv) * D]; q and k heads (adjacent in each row) leave the
        # GEMM epilogue already rotated by RoPE
        if hd == 128:
            qkv = ops.linear_rowscale(x2, w["wqkv_n"], inv1, rope=((hq + hkv) * hd, S, cfg.rope_theta))
        else:
            qkv = ops.linear_rowscale(x2, w["wqkv_n"], inv1)
            ops.rope_(qkv[:, : (hq + hkv) * hd].view(T, hq + hkv, hd), cfg.rope_theta, seq_len=S)
        q = qkv[:, : hq * hd].view(T, hq, hd)
        k = qkv[:, hq * hd: (hq + hkv) * hd].view(T, hkv, hd)
        v = qkv[:, (hq + hkv) * hd:].view(T, hkv, hd)
        mk("qkv")
        as4 = lambda t: t.view(B, S, t.shape[1], hd).transpose(1, 2)     # noqa: E731  [B, H, S, D] views
        attn = torch.empty(T, hq, hd, device=x.device, dtype=x.dtype)
        ops.fmha_fwd(as4(q), as4(k), as4(v), None, hd ** -0.5, 1, out=as4(attn))
        mk("attention")
        if self.comm == "nvls" and self.world > 1:
            x1, inv2 = self._nvls(0, T, d, x.dtype, x.device, True)(attn.view(T, hq * hd), w["wo"], x2, cfg.eps)
            mk("o_proj")
            mk("norm2")  # the residual add and the statistics ran inside the reduction
            if events is not None:
                events[0].record()
            g = ops.linear_rowscale(x1, w["w_gate_up_n"], inv2, swiglu=True)
            if events is not None:
                events[1].record()
            mk("gate_up")
            y, _ = self._nvls(1, T, d, x.dtype, x.device, False)(g, w["w_down"], x1, cfg.eps)
            y = y.clone().view(B, S, d)  # the symmetric buffer is rewritten by the next call
            mk("down")
            return y
        if self.comm in ("pipe", "nvls_pipe") and self.world > 1:
            # ``events`` bracket the whole pipelined post-attention part here (its GEMMs and
            # all-reduces interleave, so no single kernel can be bracketed)
            if events is not None:
                events[0].record()
            post = self._post_attention_pipelined if self.comm == "pipe" else self._post_attention_nvls_pipelined
            y = post(attn.view(T, hq * hd), x2).view(B, S, d)
            if events is not None:
                events[1].record()
            mk("post_attention")
            return y
        o = self._row_parallel(attn.view(T, hq * hd), w["wo"], 0, mark=mark)  # row-parallel partial -> sum
        mk("o_proj")
        inv2, x1 = ops.rms_stats(o, cfg.eps, residual=x2)               # x1 = x + o, 1/rms(x1)
        mk("norm2")
        if events is not None:
            events[0].record()
        g = ops.linear_rowscale(x1, w["w_gate_up_n"], inv2, swiglu=True)  # SwiGLU(rmsnorm(x1) W^T) [T, ff_local]
        if events is not None:
            events[1].record()
        mk("gate_up")
        # down projection + residual (in the GEMM epilogue on one rank, and on rank 0 with NCCL)
        y = self._row_parallel(g, w["w_down"], 1, resid=x1, mark=mark).view(B, S, d)
        mk("down")
        return y
