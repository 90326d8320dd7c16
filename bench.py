"""Benchmark of the fused operators on B200 — prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload (the headline): the SwiGLU MLP at the Llama-3-8B shape, bf16,
per GPU X[8192, 4096], W_gate/W_up [14336, 4096] (packed [W_gate; W_up]),
W_down [4096, 14336]; one step = gko::gemm_swiglu (one fused tcgen05 kernel)
followed by the down-projection GEMM (one tcgen05 kernel). Multi-GPU runs are
token-sharded with replicated weights (weak scaling: 8192 tokens per GPU, no
data-path collective); N > 1 is launched by torchrun, one rank per GPU.

Other workloads (for measurement; the default line uses swiglu):
  addmm_gelu   X[8192, 4096] @ W[14336, 4096]^T + b, exact GELU
  fmha_causal  causal attention B=8 H=32 S=4096 D=128 in [B, S, H, D] (heads sharded at N > 1)
  fmha_varlen  GQA varlen causal, Hq=64 Hkv=8 D=128, 16 sequences L ~ U[512, 8192] (seed 0)
  fmha_bwd     attention backward of the fmha_causal configuration
  swiglu_train forward + backward of the fused gate/up SwiGLU (training form) at the Llama-3-8B shape
  tp_block     Llama-3-70B block prefill B=4 S=4096, tensor parallel over the ranks

Timing: W untimed warm-up steps, then K steps between a barrier +
synchronize on both sides, timed with CUDA events on the launching stream;
the max over ranks is reported. Inputs are larger than the 126 MB L2 (no
flush needed). ``e2e`` repeats the step through the public operator API with
the activations copied in from pinned host memory and the result copied back
inside the timed region. ``--impl reference`` times the CPU restatement of the
reference's eager path on the host cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
TRAFFIC_FILE = REPO / "profiles" / "traffic.txt"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "fused-kernel TFLOP/s"
# --small: the attention workloads at B=4, H=16 (inputs still > L2), for full ncu captures
SMALL = False
# --tp-comm: how the tensor-parallel block sums its row-parallel outputs ("fused": inside the
# GEMM over NVLink; "nccl": GEMM then NCCL all-reduce; "nvls": NVSwitch reduction of row slices
# fused with the residual and statistics; "pipe": token-chunk pipeline of NCCL all-reduces;
# "nvls_pipe": token-chunk pipeline of the NVSwitch reductions; "auto": per rank count)
TP_COMM = "auto"
# --tp-chunks / --tp-comm-sms: token chunks of the pipelined form and the SMs its GEMMs leave free
TP_CHUNKS = 4
TP_COMM_SMS = 16


# --------------------------------------------------------------------------- helpers
def peaks():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return p, "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


def traffic_per_launch(kernel_key: str):
    """DRAM bytes (read + write) per launch of a kernel, from the committed ncu summary."""
    try:
        for line in TRAFFIC_FILE.read_text().splitlines():
            parts = line.split()
            if parts and parts[0] == kernel_key:
                for p in parts[1:]:
                    if p.startswith("dram_bytes_per_launch="):
                        return float(p.split("=", 1)[1])
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, settle_s: float = 0.3):
        self.proc = None
        self.out = None
        self.settle_s = settle_s
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            sel = str(device_index)
        self.cmd = ["nvidia-smi", "-i", sel, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "100"]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            if self.settle_s > 0:
                time.sleep(self.settle_s)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.out.strip().splitlines():
            cols = [c.strip() for c in line.split(",")]
            if len(cols) < 7:
                continue
            try:
                sm.append(float(cols[0]))
                smax.append(float(cols[1]))
            except ValueError:
                continue
            for name, val in zip(names, cols[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        busy = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    from evocompile_b200.shard import max_over_ranks as m

    return m(v)


# --------------------------------------------------------------------------- workloads
class SwigluMLP:
    name = "swiglu"
    dominant = "swiglu_gateup"
    last_out = None  # the result of the last timed step

    def close(self):
        """Release this workload's device memory before the next one is built."""
        self.__dict__.clear()

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops

        self.ops = ops
        self.T, self.D, self.H = 8192, 4096, 14336
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        self.x = torch.randn(self.T, self.D, device=dev, generator=g).to(torch.bfloat16)
        self.wgu = (torch.randn(2 * self.H, self.D, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.wd = (torch.randn(self.D, self.H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.flop_gateup = 2.0 * self.T * self.D * 2 * self.H
        self.flop_step = self.flop_gateup + 2.0 * self.T * self.H * self.D
        self.launches_per_step = 2
        self.config = {
            "workload": "swiglu_mlp llama3-8b shape: X[8192,4096] bf16, W_gate/W_up[14336,4096] packed [28672,4096], "
                        "W_down[4096,14336]; step = fused gate/up+SwiGLU kernel + down-proj GEMM",
            "inputs": "synthetic: weights N(0,0.02) at Llama-3-8B MLP shapes, X ~ N(0,1)",
            "tokens_per_gpu": self.T, "global_batch": self.T * world, "seq_len": None,
            "parallelism": f"dp{world} (token-sharded, weights replicated)",
            "l2": "operands 0.64 GB per GPU > 126 MB L2; no flush",
        }

    def step(self, ev=None):
        if ev is not None:
            ev[0].record()
        h = self.ops.linear_swiglu(self.x, self.wgu)
        if ev is not None:
            ev[1].record()
        return self.ops.linear(h, self.wd)

    # public-API end to end: pinned host inputs and the computation on their device copies
    def e2e_setup(self):
        from evocompile_b200.kernels import gemm_swiglu

        return [self.x.cpu().pin_memory()], (lambda d: gemm_swiglu.swiglu_mlp(d[0], self.wgu, self.wd))

    def torch_reference(self):
        import torch.nn.functional as F

        def mlp(x, wgu, wd):
            g, u = F.linear(x, wgu).chunk(2, dim=-1)
            return F.linear(F.silu(g) * u, wd)

        return mlp, (self.x, self.wgu, self.wd)

    def cpu_sample(self):
        """512-token sample of the same MLP for the CPU restatement (fp32)."""
        import oracle

        xs = self.x[:512].float().cpu()
        wgu, wd = self.wgu.float().cpu(), self.wd.float().cpu()
        flops = 2.0 * 512 * self.D * 2 * self.H + 2.0 * 512 * self.H * self.D
        return (lambda: oracle.swiglu_mlp(xs, wgu, wd)), flops, \
            "512 of the 8192 tokens through the full MLP (fp32 oracle restating _eager_gemm_swiglu + F.linear)"


class AddmmGelu(SwigluMLP):
    name = "addmm_gelu"
    dominant = "addmm_gelu"

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops

        self.ops = ops
        self.T, self.D, self.N = 8192, 4096, 14336
        g = torch.Generator(device=dev).manual_seed(2000 + rank)
        self.x = torch.randn(self.T, self.D, device=dev, generator=g).to(torch.bfloat16)
        self.w = (torch.randn(self.N, self.D, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.b = (torch.randn(self.N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.flop_gateup = self.flop_step = 2.0 * self.T * self.D * self.N
        self.launches_per_step = 1
        self.config = {"workload": "addmm_gelu bf16: X[8192,4096] W[14336,4096] b[14336], exact GELU",
                       "tokens_per_gpu": self.T, "global_batch": self.T * world,
                       "parallelism": f"dp{world} (token-sharded)", "l2": "operands > L2; no flush"}

    def step(self, ev=None):
        if ev is not None:
            ev[0].record()
        out = self.ops.addmm_act(self.b, self.x, self.w.t())
        if ev is not None:
            ev[1].record()
        return out

    def e2e_setup(self):
        from evocompile_b200.kernels import addmm_gelu

        addmm_gelu.register()
        return [self.x.cpu().pin_memory()], (lambda d: torch.ops.gko.addmm_gelu(self.b, d[0], self.w.t()))

    def torch_reference(self):
        import torch.nn.functional as F

        return (lambda x, w, b: F.gelu(F.linear(x, w, b))), (self.x, self.w, self.b)

    def cpu_sample(self):
        import oracle

        xs, w, b = self.x[:512].float().cpu(), self.w.float().cpu(), self.b.float().cpu()
        return (lambda: oracle.addmm_gelu(b, xs, w.t())), 2.0 * 512 * self.D * self.N, "512 of 8192 rows (fp32 oracle)"


class FmhaCausal(SwigluMLP):
    name = "fmha_causal"
    dominant = "fmha_fwd"

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops

        self.ops = ops
        B, S, H, D = (4, 4096, 16, 128) if SMALL else (8, 4096, 32, 128)
        h = H // world  # heads sharded
        self.B, self.S, self.H, self.D = B, S, h, D
        g = torch.Generator(device=dev).manual_seed(3000 + rank)
        mk = lambda: torch.randn(B, S, h, D, device=dev, generator=g).to(torch.bfloat16)  # noqa: E731
        self.qs, self.ks, self.vs = mk(), mk(), mk()
        self.q, self.k, self.v = (t.transpose(1, 2) for t in (self.qs, self.ks, self.vs))
        self.flop_gateup = self.flop_step = 4.0 * B * h * S * S * D / 2
        self.launches_per_step = 1
        self.config = {"workload": f"fmha causal bf16 B={B} H={H} S=4096 D=128 [B,S,H,D]; {h} heads per GPU",
                       "parallelism": f"heads/{world}", "l2": "q,k,v 0.8 GB > L2"}

    def step(self, ev=None):
        if ev is not None:
            ev[0].record()
        out = self.ops.fmha_fwd(self.q, self.k, self.v, None, self.D ** -0.5, 1)
        if ev is not None:
            ev[1].record()
        return out

    def e2e_setup(self):
        from evocompile_b200.kernels import fused_sdpa

        fused_sdpa.register()
        host = [t.cpu().pin_memory() for t in (self.qs, self.ks, self.vs)]
        return host, (lambda d: fused_sdpa.fused_attention(*(t.transpose(1, 2) for t in d), None, self.D ** -0.5, 1))

    def torch_reference(self):
        import torch.nn.functional as F

        return (lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True)), (self.q, self.k, self.v)

    def cpu_sample(self):
        import oracle

        q, k, v = (t[:1, :4].float().cpu() for t in (self.q, self.k, self.v))
        return (lambda: oracle.attention(q, k, v, None, self.D ** -0.5, 1)), 4.0 * 4 * self.S * self.S * self.D / 2, \
            "1 batch x 4 heads of the causal attention (fp32 oracle)"


class FmhaBackward(SwigluMLP):
    """Attention backward (gko::fused_sdpa_bwd) of the causal B=8 H=32 S=4096 D=128 configuration:
    one step = the prep, main and dq-convert kernels from the saved out / lse and a random dO."""
    name = "fmha_bwd"
    dominant = "fmha_bwd"
    compile_comparator = False

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops

        self.ops = ops
        B, S, H, D = (4, 4096, 16, 128) if SMALL else (8, 4096, 32, 128)
        h = H // world  # heads sharded
        self.B, self.S, self.H, self.D = B, S, h, D
        g = torch.Generator(device=dev).manual_seed(4000 + rank)
        mk = lambda: torch.randn(B, S, h, D, device=dev, generator=g).to(torch.bfloat16)  # noqa: E731
        self.qs, self.ks, self.vs, self.dos = mk(), mk(), mk(), mk()
        self.q, self.k, self.v, self.do = (t.transpose(1, 2) for t in (self.qs, self.ks, self.vs, self.dos))
        if dev.type == "cuda":
            self.out, self.lse = ops.fmha_fwd(self.q, self.k, self.v, None, D ** -0.5, 1)
        self.flop_gateup = self.flop_step = 2.5 * 4.0 * B * h * S * S * D / 2
        self.launches_per_step = 3
        self.config = {"workload": f"fmha backward causal bf16 B={B} H={H} S=4096 D=128 [B,S,H,D]; {h} heads per GPU; "
                                   "step = prep + main + dq-convert kernels (dq, dk, dv from q, k, v, out, lse, dO)",
                       "flop": "2.5 x the forward's causal FLOP (5 GEMMs of S^2 D / 2 per head)",
                       "parallelism": f"heads/{world}", "l2": "q,k,v,out,dO 1.3 GB > L2"}

    def step(self, ev=None):
        if ev is not None:
            ev[0].record()
        g = self.ops.fmha_bwd(self.q, self.k, self.v, None, self.out, self.lse, self.do, self.D ** -0.5, 1)
        if ev is not None:
            ev[1].record()
        return g

    def e2e_setup(self):
        from evocompile_b200.kernels import fused_sdpa

        fused_sdpa.register()
        dense = (self.qs, self.ks, self.vs, self.out.transpose(1, 2).contiguous(), self.dos)
        host = [t.cpu().pin_memory() for t in dense] + [self.lse.cpu().pin_memory()]

        def bwd(d):
            q, k, v, o, do = (t.transpose(1, 2) for t in d[:5])
            return torch.ops.gko.fused_sdpa_bwd(q, k, v, q.new_empty((0,)), o, d[5], do, self.D ** -0.5, 1, 0, 0.0)

        return host, bwd

    def torch_reference(self):
        import torch.nn.functional as F

        q, k, v = (t.detach().requires_grad_(True) for t in (self.q, self.k, self.v))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        do = self.do
        return (lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)), ()

    def cpu_sample(self):
        import oracle

        q, k, v, do = (t[:1, :1].float().cpu() for t in (self.q, self.k, self.v, self.do))
        return (lambda: oracle.attention_bwd(q, k, v, do, None, self.D ** -0.5, 1)), \
            2.5 * 4.0 * self.S * self.S * self.D / 2, "1 batch x 1 head of the causal attention backward (fp32 oracle, autograd)"


class SwigluTrain(SwigluMLP):
    """Training step of the fused gate/up SwiGLU (Llama-3-8B MLP shape): forward through
    gko::gemm_swiglu_aux (the kernel also writes the gate/up pre-activations) and backward
    from them (swiglu_bwd kernel, dX and dW on the tensor-core GEMM) — no recomputed
    forward GEMM. FLOP = 3 x the forward's 2 M D 2H."""
    name = "swiglu_train"
    dominant = "swiglu_gateup"
    traffic_key = "swiglu_gateup_aux"  # forward kernel also writes the pre-activation
    compile_comparator = False

    def __init__(self, dev, world, rank):
        super().__init__(dev, world, rank)
        from evocompile_b200.kernels import gemm_swiglu

        gemm_swiglu.register()
        self.api = gemm_swiglu
        self.xg = self.x.detach().clone().requires_grad_(True)
        self.wg = self.wgu.detach().clone().requires_grad_(True)
        g = torch.Generator(device=dev).manual_seed(1500 + rank)
        self.dy = torch.randn(self.T, self.H, device=dev, generator=g).to(torch.bfloat16)
        self.flop_step = 3.0 * self.flop_gateup
        self.launches_per_step = 4  # gate/up + aux, swiglu_bwd, dX GEMM, dW GEMM
        self.config = dict(self.config, workload="swiglu training step, llama3-8b shape: X[8192,4096] bf16, "
                           "W_gate/W_up packed [28672,4096]; step = fused gate/up forward saving gate/up + "
                           "backward (dX, dW) without recomputing the forward GEMM")

    def _fwd_bwd(self, fn):
        self.xg.grad = None
        self.wg.grad = None
        fn(self.xg, self.wg).backward(self.dy)
        return self.xg.grad

    def step(self, ev=None):
        # the events bracket the forward gate/up kernel (the record's dominant kernel: it also
        # writes the pre-activation); the backward launches follow outside them
        self.xg.grad = None
        self.wg.grad = None
        if ev is not None:
            ev[0].record()
        y = self.api.apply_train(self.xg, self.wg)
        if ev is not None:
            ev[1].record()
        y.backward(self.dy)
        return self.xg.grad

    def e2e_setup(self):
        api = self.api
        wg = self.wg
        dy = self.dy

        def train(d):
            x = d[0].detach().requires_grad_(True)  # a leaf view; the pipeline's buffer stays grad-free
            wg.grad = None
            api.apply_train(x, wg).backward(dy)
            return x.grad

        return [self.x.cpu().pin_memory()], train

    def torch_reference(self):
        import torch.nn.functional as F

        def eager(x, w):
            g, u = F.linear(x, w).chunk(2, dim=-1)
            return F.silu(g) * u

        return (lambda: self._fwd_bwd(eager)), ()

    def extra_arms(self):
        return {"gko_recompute_backward": lambda: self._fwd_bwd(torch.ops.gko.gemm_swiglu)}

    def cpu_sample(self):
        import oracle

        xs = self.x[:256].float().cpu().requires_grad_(True)
        w = self.wgu.float().cpu().requires_grad_(True)
        dy = self.dy[:256].float().cpu()

        def fn():
            xs.grad = None
            w.grad = None
            oracle.gemm_swiglu(xs, w).backward(dy)

        return fn, 3.0 * 2.0 * 256 * self.D * 2 * self.H, "256 of 8192 tokens, forward + backward (fp32 oracle autograd)"


class FmhaVarlen(SwigluMLP):
    name = "fmha_varlen"
    dominant = "fmha_varlen_fwd"

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops, shard

        self.ops = ops
        gl = torch.Generator().manual_seed(0)
        lens_all = torch.randint(512, 8193, (16,), generator=gl).tolist()
        mine = shard.balance_sequences(lens_all, world)[rank]
        self.lens = [lens_all[i] for i in mine]
        self.cu = torch.tensor(shard.cu_seqlens(self.lens), dtype=torch.int32, device=dev)
        T = int(sum(self.lens))
        g = torch.Generator(device=dev).manual_seed(4000 + rank)
        self.q = torch.randn(T, 64, 128, device=dev, generator=g).to(torch.bfloat16)
        self.k = torch.randn(T, 8, 128, device=dev, generator=g).to(torch.bfloat16)
        self.v = torch.randn(T, 8, 128, device=dev, generator=g).to(torch.bfloat16)
        self.flop_gateup = self.flop_step = float(sum(2 * 64 * 128 * L * L for L in self.lens))
        self.launches_per_step = 1
        self.config = {"workload": "fmha varlen causal GQA bf16 Hq=64 Hkv=8 D=128, 16 seqs L~U[512,8192] seed 0",
                       "tokens_this_rank": T, "seqs_this_rank": len(self.lens),
                       "parallelism": f"sequences/{world} token-balanced", "l2": "q,k,v > L2"}

    def step(self, ev=None):
        if ev is not None:
            ev[0].record()
        out = self.ops.fmha_varlen_fwd(self.q, self.k, self.v, self.cu, self.cu, max(self.lens), max(self.lens),
                                       128 ** -0.5, 1)
        if ev is not None:
            ev[1].record()
        return out

    def e2e_setup(self):
        from evocompile_b200.kernels import fused_sdpa

        fused_sdpa.register()
        host = [t.cpu().pin_memory() for t in (self.q, self.k, self.v)]
        return host, (lambda d: torch.ops.gko.fmha_varlen_fwd(*d, self.cu, self.cu, max(self.lens), max(self.lens),
                                                              128 ** -0.5, 1)[0])

    def torch_reference(self):
        """Per-sequence causal GQA SDPA over the packed tensors (torch has no varlen SDPA API)."""
        import torch.nn.functional as F

        bounds = list(zip(self.cu.tolist()[:-1], self.cu.tolist()[1:]))

        def ref(q, k, v):
            outs = []
            for s, e in bounds:
                qs, ks, vs = (t[s:e].transpose(0, 1)[None] for t in (q, k, v))
                outs.append(F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, enable_gqa=True)[0]
                            .transpose(0, 1))
            return torch.cat(outs)

        return ref, (self.q, self.k, self.v)

    def cpu_sample(self):
        import oracle

        L = min(self.lens)
        cu = torch.tensor([0, L], dtype=torch.int32)
        q, k, v = (t[:L].float().cpu() for t in (self.q, self.k, self.v))
        return (lambda: oracle.attention_varlen(q, k, v, cu, cu, 128 ** -0.5, 1)), 2.0 * 64 * 128 * L * L, \
            f"the shortest sequence (L={L}) of this rank (fp32 oracle)"


class TPBlockWorkload(SwigluMLP):
    """Llama-3-70B-shaped block prefill, B=4 S=4096 (T=16384), tensor-parallel over the ranks."""

    name = "tp_block"
    dominant = "swiglu_gateup"
    traffic_key = "swiglu_gateup_llama3_70b"  # d_model 8192, d_ff 28672 per rank
    scaling = "strong"

    def __init__(self, dev, world, rank):
        from evocompile_b200 import ops
        from evocompile_b200.block import BlockConfig, TPBlock, init_weights, shard_weights

        self.ops = ops
        self.cfg = BlockConfig()
        self.B, self.S = 4, 4096
        self.world = world
        self.rank = rank
        full = init_weights(self.cfg, dev, torch.bfloat16, seed=7)
        self.full = full if world == 1 else None
        # rank 0 keeps an fp32 host copy of the full weights for the CPU leg (oracle timing and parity)
        self.w_host = {k: v.float().cpu() for k, v in full.items()} if rank == 0 else None
        group = None
        if world > 1:
            import torch.distributed as dist

            group = dist.group.WORLD
        self.block = TPBlock(shard_weights(full, self.cfg, rank, world), self.cfg, group, comm=TP_COMM,
                             chunks=TP_CHUNKS, comm_sms=TP_COMM_SMS)
        if world > 1:
            del full
            torch.cuda.empty_cache()
        g = torch.Generator(device=dev).manual_seed(8)  # same activations on every rank (replicated input)
        self.x = torch.randn(self.B, self.S, self.cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
        T, hd = self.B * self.S, self.cfg.head_dim
        self.flop_step = self.cfg.flops(T, self.S)
        ff_l = self.cfg.d_ff // world
        self.flop_gateup = 2.0 * T * self.cfg.d_model * 2 * ff_l
        if world > 1:
            self.traffic_key = None  # the captured shape is TP1's; a rank's gate/up is 1/world of it
        if self.block.comm in ("pipe", "nvls_pipe") and world > 1:
            # the step's events bracket the pipelined post-attention part: o-projection, gate/up
            # and down GEMMs with their all-reduces
            self.dominant = "post_attention_pipelined"
            self.flop_gateup += 2.0 * T * (self.cfg.n_heads // world) * hd * self.cfg.d_model \
                + 2.0 * T * ff_l * self.cfg.d_model
        self.launches_per_step = 7  # rms stats, qkv gemm (+ RoPE), fmha, o gemm, rms stats, gate/up, down
        self.config = {
            "workload": "llama3-70b block prefill bf16: d_model 8192, 64 q / 8 kv heads, D 128, d_ff 28672, "
                        "B=4 S=4096; RMSNorm -> QKV -> RoPE(5e5) -> causal GQA FMHA -> o-proj -> residual -> "
                        "RMSNorm -> SwiGLU -> down -> residual",
            "inputs": "synthetic: weights N(0,0.02) at Llama-3-70B block shapes, x ~ N(0,1)",
            "global_batch": self.B, "seq_len": self.S, "tokens": T,
            "parallelism": f"tp{world} (column-parallel QKV / gate-up, row-parallel o / down; row-parallel sums: "
                           + ("none" if world == 1 else {
                               "fused": "inside the GEMM over NVLink (multicast reduction)",
                               "nccl": "NCCL all-reduce after each GEMM",
                               "pipe": f"NCCL all-reduces of {self.block.chunks} token chunks overlapping the "
                                       f"next chunks' GEMMs",
                               "nvls": "NVSwitch multicast reduction of row slices fused with the residual "
                                       "add and RMS statistics",
                               "nvls_pipe": f"NVSwitch reductions (residual add and RMS statistics fused) of "
                                            f"{self.block.chunks} token chunks overlapping the next chunks' "
                                            f"GEMMs"}[self.block.comm]) + ")",
            "l2": "weights 1.7 GB / tp, activations > L2; no flush",
        }

    def step(self, ev=None):
        # the events bracket the fused gate/up + SwiGLU kernel inside the block
        return self.block.forward(self.x, events=ev)

    def phases(self, steps, world):
        """Device ms per step of each phase of the block (CUDA events at every phase boundary on
        the launching stream, averaged over ``steps`` steps, max over ranks). With NCCL the
        row-parallel projections split into their GEMM and their all-reduce."""
        marks = []

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            marks.append((name, e))

        for _ in range(steps):
            self.block.forward(self.x, mark=mark)
        torch.cuda.synchronize()
        # an interval that ends at a projection's mark and starts at that GEMM's own mark is its all-reduce
        out = {}
        names = [n for n, _ in marks]
        for i in range(1, len(marks)):
            name, prev = names[i], names[i - 1]
            if name == "start":
                continue
            key = f"{name}_allreduce" if prev == f"{name}_gemm" else name
            out[key] = out.get(key, 0.0) + marks[i - 1][1].elapsed_time(marks[i][1])
        keys = sorted(out)
        vals = [out[k] / steps for k in keys]
        if world > 1:
            import torch.distributed as dist

            t = torch.tensor(vals, dtype=torch.float64, device=self.x.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            vals = t.tolist()
        return dict(zip(keys, vals))

    def cpu_check(self):
        """Parity of this run's output (the last timed step, rank 0) against the oracle on the
        first 512 tokens of sequence 0: rows of a causal block depend only on their prefix, so
        the oracle's 512-token block gives exactly those rows. Reported as max|err| / max|ref| of
        the block output and of the block's update (output - x)."""
        import oracle

        torch.set_num_threads(os.cpu_count() or 1)
        P = 512
        xs = self.x[:1, :P].float().cpu()
        t0 = time.perf_counter()
        ref = oracle.llama_block(xs, self.w_host, self.cfg)
        dt = time.perf_counter() - t0
        got = self.last_out[:1, :P].float().cpu()
        rel = ((got - ref).abs().max() / ref.abs().max()).item()
        d_got, d_ref = got - xs, ref - xs
        rel_d = ((d_got - d_ref).abs().max() / d_ref.abs().max()).item()
        return {"parity": {"rel_err": rel, "rel_err_delta": rel_d, "tol": 2e-2, "ok": rel <= 2e-2,
                           "rows": f"sequence 0, tokens [0, {P}) of the timed run's output (rank 0)",
                           "oracle": "oracle.llama_block, fp32 on the host cores, from the same bf16 weights",
                           "oracle_s": dt},
                "comm": self.block.comm if self.world > 1 else "none",
                "nccl": {"backend": "nccl", "ranks": self.world} if self.world > 1 else None}

    def e2e_setup(self):
        return [self.x.cpu().pin_memory()], (lambda d: self.block.forward(d[0]))

    def torch_reference(self):
        import torch.nn.functional as F

        if self.full is None:
            return None, None
        cfg, w = self.cfg, self.full
        hd = cfg.head_dim

        def rms(t, wt):
            tf = t.float()
            return (tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + cfg.eps)).to(t.dtype) * wt

        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=self.x.device).float() / hd))
        ang = torch.arange(self.S, device=self.x.device).float()[:, None] * inv[None]
        cos = torch.cat([ang.cos(), ang.cos()], -1).to(torch.bfloat16)[None, :, None, :]
        sin = torch.cat([ang.sin(), ang.sin()], -1).to(torch.bfloat16)[None, :, None, :]

        def rot(t):
            t1, t2 = t[..., : hd // 2], t[..., hd // 2:]
            return t * cos + torch.cat([-t2, t1], -1) * sin

        def blk(x):
            B, S, d = x.shape
            h = rms(x, w["attn_norm"])
            q = rot(F.linear(h, w["wq"]).view(B, S, cfg.n_heads, hd)).transpose(1, 2)
            k = rot(F.linear(h, w["wk"]).view(B, S, cfg.n_kv_heads, hd)).transpose(1, 2)
            v = F.linear(h, w["wv"]).view(B, S, cfg.n_kv_heads, hd).transpose(1, 2)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            x1 = x + F.linear(o.transpose(1, 2).reshape(B, S, d), w["wo"])
            h2 = rms(x1, w["mlp_norm"])
            return x1 + F.linear(F.silu(F.linear(h2, w["w_gate"])) * F.linear(h2, w["w_up"]), w["w_down"])

        return blk, (self.x,)

    def cpu_sample(self):
        import oracle

        cfg, w = self.cfg, self.w_host
        xs = self.x[:1, :512].float().cpu()
        return (lambda: oracle.llama_block(xs, w, cfg)), cfg.flops(512, 512), \
            "one 512-token sequence through the full-width block (fp32 oracle)"


class E2EPipeline:
    """End to end through the public API, host memory to host memory, pipelined like a serving
    loop: two slots of device inputs; step i uploads its inputs on one copy stream while the
    previous step computes, and downloads its result on a second copy stream while the next
    step computes. Every step moves all of its inputs from pinned host memory and all of its
    outputs back; the timed region ends when the last download has finished."""

    def __init__(self, host_inputs, compute, dev):
        self.host_in = host_inputs
        self.compute = compute
        self.dev_in = [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host_inputs] for _ in range(2)]
        self.up, self.down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.host_out = [None, None]
        self.h2d_bytes = sum(h.numel() * h.element_size() for h in host_inputs)
        self.d2h_bytes = 0

    def begin(self, start):
        self.up.wait_event(start)
        self.down.wait_event(start)

    def step(self, i):
        s = i % 2
        cur = torch.cuda.current_stream()
        with torch.cuda.stream(self.up):
            self.up.wait_event(self.consumed[s])  # the compute two steps back has read this slot
            for d, h in zip(self.dev_in[s], self.host_in):
                d.copy_(h, non_blocking=True)
            self.loaded[s].record(self.up)
        cur.wait_event(self.loaded[s])
        out = self.compute(self.dev_in[s])
        outs = out if isinstance(out, (tuple, list)) else (out,)
        self.consumed[s].record(cur)
        self.computed[s].record(cur)
        if self.host_out[s] is None:  # first use of the slot (a warm-up step)
            self.host_out[s] = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
            self.d2h_bytes = sum(o.numel() * o.element_size() for o in outs)
        with torch.cuda.stream(self.down):
            self.down.wait_event(self.computed[s])
            for hb, o in zip(self.host_out[s], outs):
                hb.copy_(o, non_blocking=True)
                o.record_stream(self.down)

    def join(self):
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.up)
        cur.wait_stream(self.down)


WORKLOADS = {c.name: c for c in (SwigluMLP, SwigluTrain, AddmmGelu, FmhaCausal, FmhaBackward, FmhaVarlen,
                                  TPBlockWorkload)}


# --------------------------------------------------------------------------- arms
def time_cpu(fn, flops, budget_s=10.0, max_reps=20):
    fn()  # warm
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps == 0 or time.perf_counter() - t0 < budget_s):
        fn()
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return flops / dt / 1e12, dt, reps


def run_reference(args):
    """The reference's eager path restated on the host CPU cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    wl_cls = WORKLOADS[args.workload]
    # built on the CPU from the same seeds; nothing of this arm touches the GPU
    wl = wl_cls(torch.device("cpu"), 1, 0)
    fn, flops, sample = wl.cpu_sample()
    for _ in range(max(args.warmup, 0)):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = flops / (ms / 1e3) / 1e12
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(wl.config, sample=sample),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# seconds of warm-up work before a timed region: a record starts after the host-only CPU leg
# of the previous one, and under the 1 kW power cap the SM clock needs some seconds of load to
# settle (the clocks the sampler saw are in each record's ``clocks``)
WARM_S = 3.0
# seconds of continuous warm-up of each comparator arm (torch eager, torch.compile, our step again)
# right before its timed steps
COMPARATOR_WARM_S = 2.0


def _warm(step, warmup, world, dev, min_s=1.0):
    """W warm-up steps, then more until about ``min_s`` seconds of work have run (after a stretch
    of host-only work the GPU's clocks take a while to come back up). Every rank runs the same
    count: a step of the tensor-parallel block holds collectives."""
    t0 = time.perf_counter()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    per_step = (time.perf_counter() - t0) / max(1, warmup)
    more = int(max_over_ranks(max(0.0, min_s - per_step * warmup) / max(per_step, 1e-6), world))
    for _ in range(more):
        step()
    torch.cuda.synchronize(dev)


def _timed_region(wl, steps, warmup, world, local, dev):
    """W warm-up steps, then K steps between barrier + synchronize, CUDA events on the launching
    stream; per-step events bracket the dominant kernel. Returns max-over-ranks step and kernel ms."""
    from evocompile_b200 import _lib

    stream = torch.cuda.current_stream(dev)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the clock sampler starts before the warm-up: nvidia-smi's start-up then overlaps GPU work
    # instead of leaving the GPU idle (and its clocks falling) right before the timed steps
    with ClockSampler(local, settle_s=0.0) as clocks:
        _warm(wl.step, warmup, world, dev, min_s=WARM_S)
        if _lib.read_status(dev):
            raise RuntimeError(f"{wl.name}: kernel timeout during warm-up")
        barrier(world)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for i in range(steps):
            wl.last_out = wl.step(kev[i])
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / steps, world)
    return ms, kern_ms, clocks.summary(), _lib.read_status(dev)


def _e2e_record(wl, steps, warmup, world, dev, scale):
    """End to end through the public op API, pinned host memory to pinned host memory."""
    host, fn = wl.e2e_setup()
    pipe = E2EPipeline(host, fn, dev)
    stream = torch.cuda.current_stream(dev)
    n = max(5, min(steps, 50))
    # warm-up: untimed pipelined steps for at least a second and at least the timed count (the
    # first pipelined host copies of a process run well below the link's rate for a while)
    counter = iter(range(1 << 30))
    _warm(lambda: pipe.step(next(counter)), max(2, warmup, n), world, dev)
    pipe.join()
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    pipe.begin(a)
    for i in range(n):
        pipe.step(i)
    pipe.join()
    b.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    local_ms = a.elapsed_time(b) / n
    pipe_ms = max_over_ranks(local_ms, world)
    h2d, d2h = pipe.h2d_bytes, pipe.d2h_bytes
    del pipe, host, fn
    return {"value": scale * wl.flop_step / (pipe_ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": pipe_ms, "steps": n,
            # this rank's host link rate over the pipelined steps: at N > 1 all ranks share one
            # host's PCIe / memory bandwidth, which bounds e2e before any kernel does
            "h2d_gbs_per_rank": h2d / (local_ms / 1e3) / 1e9, "d2h_gbs_per_rank": d2h / (local_ms / 1e3) / 1e9}


def _comparators(wl, steps, dev):
    """torch eager and torch.compile of the harness-equivalent module on the same GPU, and our
    step again (``gko_repeat``), each timed like our arm: COMPARATOR_WARM_S seconds of its own
    continuous warm-up, then K steps between CUDA events. Under the power cap a short burst after
    other work runs at higher clocks than sustained load, so every arm is measured sustained, as
    the record's ``value`` is."""
    stream = torch.cuda.current_stream(dev)
    comparators = {}
    fn, fargs = wl.torch_reference()
    arms = {}
    if fn is not None:
        arms["torch_eager"] = lambda: fn(*fargs)
        if getattr(wl, "compile_comparator", True):
            try:
                cfn = torch.compile(fn)
                arms["torch_compile"] = lambda: cfn(*fargs)
            except Exception as e:  # noqa: BLE001
                comparators["torch_compile"] = {"error": repr(e)[:200]}
    arms["gko_repeat"] = lambda: wl.step()
    if hasattr(wl, "extra_arms"):
        arms.update(wl.extra_arms())
    for name, f in list(arms.items()):
        try:
            for _ in range(3):
                f()
            torch.cuda.synchronize(dev)
        except Exception as e:  # noqa: BLE001
            comparators[name] = {"error": repr(e)[:200]}
            arms.pop(name)
    for name, f in arms.items():
        _warm(f, 3, 1, dev, min_s=COMPARATOR_WARM_S)
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        for _ in range(steps):
            f()
        x1.record(stream)
        torch.cuda.synchronize(dev)
        t = x0.elapsed_time(x1) / steps
        comparators[name] = {"ms_per_step": t, "tflops": wl.flop_step / t / 1e9, "warm_s": COMPARATOR_WARM_S}
    torch._dynamo.reset()
    return comparators


def _cpu_leg(wl, budget_s):
    """The oracle on a bounded sample of the workload on the host cores (rank 0): the CPU
    baseline, and for workloads that define ``cpu_check`` the parity of the GPU result."""
    torch.set_num_threads(os.cpu_count() or 1)
    fn, flops, sample = wl.cpu_sample()
    tf, dt, reps = time_cpu(fn, flops, budget_s=budget_s)
    cpu = {"value": tf, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
           "sample": f"{sample}; {reps} reps, {dt * 1e3:.1f} ms each"}
    return cpu


def measure(wl, args, world, rank, local, dev, compare, cpu, cpu_budget_s=10.0):
    """Every figure of one workload's record (identical collective sequence on every rank)."""
    from evocompile_b200 import _lib

    ms, kern_ms, clocks, status = _timed_region(wl, args.steps, args.warmup, world, local, dev)
    extra = {}
    if hasattr(wl, "phases"):
        extra["phases_ms"] = wl.phases(args.steps, world)
    scale = 1 if getattr(wl, "scaling", "weak") == "strong" else world  # strong: flop_step is the whole job
    e2e = _e2e_record(wl, args.steps, args.warmup, world, dev, scale)
    comparators = _comparators(wl, args.steps, dev) if (world == 1 and compare) else None
    cpu_rec = None
    if rank == 0 and hasattr(wl, "cpu_check"):
        extra.update(wl.cpu_check())
    if rank == 0 and world == 1 and cpu:
        cpu_rec = _cpu_leg(wl, cpu_budget_s)
    status |= _lib.read_status(dev)
    pk, pk_src = peaks()
    peak = pk["bf16_tflops"]
    value = scale * wl.flop_step / (ms / 1e3) / 1e12
    achieved = wl.flop_gateup / (kern_ms / 1e3) / 1e12
    traffic = traffic_per_launch(getattr(wl, "traffic_key", wl.dominant))
    rec = {
        "value": value, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world,
        "scaling": getattr(wl, "scaling", "weak"), "config": wl.config,
        "pct_of_peak": value / (world * peak),
        "tokens_per_s": (wl.B * wl.S / (ms / 1e3)) if getattr(wl, "scaling", "weak") == "strong"
        else (world * wl.T / (ms / 1e3) if hasattr(wl, "T") else None),
        "roofline": {"bound": "tensor", "kernel": wl.dominant, "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{pk_src} bf16 burst (MEASURED_PEAKS.json)" if pk_src == "measured"
                     else "fallback 1590 TFLOP/s", "flop_per_launch": wl.flop_gateup,
                     "avg_launch_ms": kern_ms},
        "cpu_baseline": cpu_rec,
        "e2e": e2e,
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clocks,
        "comparators": comparators,
        "kernel_status": status,
    }
    rec.update(extra)
    return rec


# the per-configuration records added to the default line: every configuration of the
# operators at its full size (sharded at N > 1 as the configuration shards)
SUB_WORKLOADS = ("addmm_gelu", "swiglu_train", "fmha_causal", "fmha_varlen", "fmha_bwd", "tp_block")


def run_ours(args):
    world, rank, local = dist_setup()
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from evocompile_b200 import _lib

    _lib.load()
    compare = not args.no_compare
    wl = WORKLOADS[args.workload](dev, world, rank)
    rec = measure(wl, args, world, rank, local, dev, compare, not args.no_cpu)
    del wl
    torch.cuda.empty_cache()

    subs = {}
    names = [] if args.no_workloads or args.workload != "swiglu" else \
        [n for n in (args.workloads.split(",") if args.workloads else SUB_WORKLOADS) if n]
    for name in names:
        sub = WORKLOADS[name](dev, world, rank)
        try:
            subs[name] = measure(sub, args, world, rank, local, dev, compare, not args.no_cpu, cpu_budget_s=5.0)
        finally:
            sub.close()
            del sub
            torch.cuda.empty_cache()

    if rank == 0:
        line = {
            "metric": METRIC, "value": rec["value"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": rec["scaling"], "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": rec["config"],
        }
        for key in ("pct_of_peak", "tokens_per_s", "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks",
                    "comparators", "kernel_status", "phases_ms", "rel_err", "rel_err_delta", "parity", "comm",
                    "nccl"):
            if key in rec:
                line[key] = rec[key]
        if subs:
            for r in subs.values():
                r.pop("n_gpus", None)
            line["workloads"] = subs
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="swiglu")
    ap.add_argument("--no-compare", action="store_true", help="skip the torch eager / torch.compile comparators")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-workloads", action="store_true",
                    help="default line without the per-configuration records (headline only)")
    ap.add_argument("--workloads", default="",
                    help=f"comma-separated per-configuration records to add (default: {','.join(SUB_WORKLOADS)})")
    ap.add_argument("--small", action="store_true",
                    help="attention workloads at B=4, H=16 (a capture-sized case for ncu --set full)")
    ap.add_argument("--tp-comm", choices=("auto", "fused", "nccl", "pipe", "nvls", "nvls_pipe"), default="auto",
                    help="tp_block: sum row-parallel outputs inside the GEMM (fused), with a blocking NCCL "
                         "all-reduce (nccl), with NCCL all-reduces of token chunks overlapping the next "
                         "chunks' GEMMs (pipe), with NVSwitch reductions of row slices (nvls) or of token "
                         "chunks overlapping the next chunks' GEMMs (nvls_pipe), or per rank count (auto)")
    ap.add_argument("--tp-chunks", type=int, default=4, help="tp_block pipe / nvls_pipe: token chunks")
    ap.add_argument("--tp-comm-sms", type=int, default=16,
                    help="tp_block pipe / nvls_pipe: SMs the GEMMs leave to the reductions")
    args = ap.parse_args()
    global SMALL, TP_COMM, TP_CHUNKS, TP_COMM_SMS
    SMALL = args.small
    TP_COMM = args.tp_comm
    TP_CHUNKS = args.tp_chunks
    TP_COMM_SMS = args.tp_comm_sms
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
