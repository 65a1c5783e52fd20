#!/usr/bin/env python
"""Benchmark of the fused decode hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload f2|f1|f4|gqa|mlp|qkv|layer|f2fp8|mlpblock]

The benchmark's five configs: C1 F1 RMSNorm -> GEMV 4096x4096 fp16; C2 F2
gate+up -> SwiGLU, Wg/Wu [11008,4096] fp16; C3 F4 MHA FlashDecode, 32 heads x
4096 tokens; C4 Llama-70B decode MLP, batch 16, bf16; C5 GQA paged FlashDecode,
batch 8, 64/8 heads, lengths ~U[1024,32768]. qkv, layer and f2fp8 are the
added rows (QKV + RoPE + cache append, a whole decode layer, fp8 weights).

A step is one pass of the fused hot path over one decode batch. The default
workload is config C2 (F2: gate+up GEMV -> SwiGLU, x [1,4096] fp16,
Wg/Wu [11008,4096] fp16 ~N(0,1)/64). With N GPUs (torchrun, one process per
GPU) the weights are column-sharded (d_ff/N rows per rank) and the all-gather
of h runs inside the GEMV kernel over NVLink peer memory (NCCL with
DBK_EXCHANGE=nccl): total work is fixed ("strong" scaling).

Reported:
  value      whole-job HBM GB/s = algorithmic bytes of a step / max-over-ranks
             device time per step (CUDA events, graph replay, weights rotated
             over replicas larger than L2 in total);
  e2e        the same metric through the public API (decodebench_b200.ops) with
             the step's activation copied in from pinned host memory and the
             result copied back, every step;
  roofline   the fused kernel's algorithmic bytes per launch / its average
             launch duration, against MEASURED_PEAKS.json's HBM copy bandwidth;
  cpu_baseline  the reference's own CPU implementation (oracle/_ref, compiled
             from its cpu_reference.cpp) on this host's cores (rank 0, N=1).
``--impl reference`` times only that CPU implementation (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "fused decode µs/step & HBM GB/s (% of B200 peak) at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------- helpers
def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_table() -> dict:
    p = ROOT / "profiles" / "dram_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons in a background thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples: list[tuple[float, int, int]] = []
        self.period = period_s
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report the absence, never fail the bench
            self.err = f"{type(e).__name__}: {e}"
        self.t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self.t.start()

    def count_between(self, t0, t1) -> int:
        return sum(1 for s in self.samples if t0 <= s[0] <= t1)

    def stop(self):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self, t0: float, t1: float) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": self.err}
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        bits = 0
        for _, _, r in win:
            bits |= r
        return {"sm_mhz": statistics.median(m for _, m, _ in win), "sm_max_mhz": self.max_mhz,
                "reasons": [n for b, n in self.REASONS.items() if bits & b and n != "gpu_idle"],
                "samples": len(win), "source": "nvml, 5 ms period, timed region"}


# ---------------------------------------------------------------- workloads
class Workload:
    """One fused decode step on this rank, with sharding over `world` ranks."""

    name = ""
    kernels_per_step = 1

    def describe(self) -> dict: ...
    def step_bytes_total(self) -> int: ...
    def launch_bytes(self) -> int: ...
    def run_kernel(self, rep: int) -> None: ...
    def exchange(self) -> None: ...
    def e2e_setup(self) -> tuple[int, int]: ...
    def e2e_step(self) -> None: ...

    with_exchange = True      # False while capturing the kernel-only (roofline) graphs
    comm = None               # decodebench_b200.comm.PeerComm when the peer exchange is on
    exchanges_per_step = 1    # shard-boundary all-gathers per step at N > 1

    def xname(self) -> str:
        return ("peer-store all-gather over NVLink (dbk_allgather)" if self.comm is not None
                else "NCCL all-gather")

    def gather_blocks(self, local, out=None):
        """[*shape] per rank -> [world, *shape] in rank order."""
        if self.comm is not None:
            return self.comm.all_gather_blocks(local, out)
        if out is None:
            out = self.t.empty(self.world, *local.shape, dtype=local.dtype, device=local.device)
        self.t.distributed.all_gather_into_tensor(out, local)
        return out

    def gather_rows(self, local, out=None):
        """[rows, n] per rank -> [rows, world * n], rank p in columns [p n, (p + 1) n)."""
        if self.comm is not None:
            return self.comm.all_gather_rows(local, out)
        rows, n = local.shape
        full = self.t.empty(self.world, rows, n, dtype=local.dtype, device=local.device)
        self.t.distributed.all_gather_into_tensor(full, local.contiguous())
        res = full.permute(1, 0, 2).reshape(rows, self.world * n)
        if out is None:
            return res
        out.copy_(res)
        return out


class F2(Workload):
    """config C2: x [1,4096] fp16, Wg/Wu [11008,4096] fp16 ~N(0,1)/64."""

    name = "f2"

    def __init__(self, rank, world, torch, d_in=4096, d_ff=11008, batch=1):
        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world = rank, world
        self.d_in, self.d_ff, self.batch = d_in, d_ff, batch
        if d_ff % world:
            raise SystemExit(f"d_ff={d_ff} does not split over {world} ranks")
        self.rows = d_ff // world
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        sc = 1.0 / math.sqrt(d_in)
        per_rep = 2 * self.rows * d_in * 2
        self.nrep = max(2, math.ceil(2 * 126e6 / per_rep)) if per_rep < 400e6 else 1
        self.nrep = min(self.nrep, 64)
        self.W = [((torch.randn(self.rows, d_in, generator=g, device=dev) * sc).half(),
                   (torch.randn(self.rows, d_in, generator=g, device=dev) * sc).half())
                  for _ in range(self.nrep)]
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(batch, d_in, generator=xg).half()
        self.x = self.x_cpu.to(dev)
        self.h_local = torch.empty(batch, self.rows, dtype=torch.float16, device=dev)
        self.h_full = torch.empty(batch, world * self.rows, dtype=torch.float16, device=dev)

    def describe(self):
        return {"workload": f"F2 gate+up GEMV -> SwiGLU, x [{self.batch},{self.d_in}] fp16, "
                            f"Wg/Wu [{self.d_ff},{self.d_in}] fp16 "
                            + ("(config C2)" if self.d_ff == 11008 else "(--rows override)"),
                "global_batch": self.batch, "d_in": self.d_in, "d_ff": self.d_ff,
                "parallelism": ("single GPU" if self.world == 1 else
                                f"tp{self.world}: d_ff column-sharded, {self.xname()} of h"),
                "weight_replicas": self.nrep,
                "l2": f"weights rotated over {self.nrep} replicas "
                      f"({self.nrep * 2 * self.rows * self.d_in * 2 / 1e6:.0f} MB per GPU > 126 MB L2)"}

    def step_bytes_total(self):
        return self.costs.gateup_swiglu_bytes(self.batch, self.d_in, self.d_ff)

    def launch_bytes(self):
        return self.costs.gateup_swiglu_bytes(self.batch, self.d_in, self.rows)

    exchanges_per_step = 0    # at N > 1 the all-gather runs inside the GEMV kernel

    def xname(self) -> str:
        return ("all-gather fused into the GEMV kernel (NVLink peer stores)"
                if self.comm is not None else "NCCL all-gather")

    def fused(self) -> bool:
        """N > 1 with the peer exchange: the all-gather runs inside the GEMV kernel."""
        return self.world > 1 and self.comm is not None and self.with_exchange

    def run_kernel(self, rep):
        Wg, Wu = self.W[rep % self.nrep]
        if self.fused():
            self.ops.gateup_swiglu(self.x, Wg, Wu, out=self.h_full, comm=self.comm)
        else:
            self.ops.gateup_swiglu(self.x, Wg, Wu, out=self.h_local)

    def exchange(self):
        if self.world > 1 and not self.fused():
            self.gather_rows(self.h_local, self.h_full)

    def torch_kernel(self, rep):
        """Library baseline: the same step with PyTorch ops (cuBLAS GEMVs)."""
        F = self.t.nn.functional
        Wg, Wu = self.W[rep % self.nrep]
        return F.silu(F.linear(self.x, Wg)) * F.linear(self.x, Wu)

    def e2e_setup(self):
        t = self.t
        self.x_host = self.x_cpu.pin_memory()
        self.out_host = t.empty(self.world * self.batch * self.rows, dtype=t.float16).pin_memory()
        self.x_dev = t.empty_like(self.x)
        self._e2e_i = 0
        return self.x_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        Wg, Wu = self.W[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.x_dev, self.x_host)
        if self.world > 1 and self.comm is not None:
            h = self.ops.gateup_swiglu(self.x_dev, Wg, Wu, out=self.h_full, comm=self.comm)
        elif self.world == 1:
            # the kernel writes h straight into the pinned host buffer
            self.ops.gateup_swiglu(self.x_dev, Wg, Wu, out=self.out_host.view(self.batch, -1))
            return
        else:
            h = self.gather_rows(self.ops.gateup_swiglu(self.x_dev, Wg, Wu, out=self.h_local))
        self.ops.stage(self.out_host, h.reshape(-1))

    # reference CPU implementation (oracle/_ref: the reference's cpu_reference.cpp)
    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.d_ff * frac_rows))
        self.cpu_rows = n
        self.cWg = (rng.standard_normal((n, self.d_in), dtype=np.float32) / math.sqrt(self.d_in)
                    ).astype(np.float16).astype(np.float32)
        self.cWu = (rng.standard_normal((n, self.d_in), dtype=np.float32) / math.sqrt(self.d_in)
                    ).astype(np.float16).astype(np.float32)
        self.cx = self.x_cpu.float().numpy()[0].copy()

    def cpu_step(self, threads):
        from oracle import oracle as O

        g = O.ref_gemv_threaded(self.cWg, self.cx, threads)
        u = O.ref_gemv_threaded(self.cWu, self.cx, threads)
        return O.swiglu_f32(g, u, use_ref=True)

    def cpu_step_bytes(self):
        return self.costs.gateup_swiglu_bytes(self.batch, self.d_in, self.cpu_rows)


class F1(F2):
    """config C1 on the GPU: RMSNorm -> GEMV, 4096 x 4096 fp16."""

    name = "f1"

    def __init__(self, rank, world, torch, d=4096, d_out=None):
        from decodebench_b200 import costs, ops

        d_out = d_out or d
        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.batch, self.d_in, self.d_ff = rank, world, 1, d, d_out
        if d_out % world:
            raise SystemExit(f"d_out={d_out} does not split over {world} ranks")
        self.rows = d_out // world
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        per_rep = self.rows * d * 2
        self.nrep = min(64, max(2, math.ceil(2 * 126e6 / per_rep)))
        self.W = [(torch.randn(self.rows, d, generator=g, device=dev) / 64).half()
                  for _ in range(self.nrep)]
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(1, d, generator=xg).half()
        self.g_cpu = torch.randn(d, generator=xg).half()
        self.x, self.gamma = self.x_cpu.to(dev), self.g_cpu.to(dev)
        self.h_local = torch.empty(1, self.rows, dtype=torch.float16, device=dev)
        self.h_full = torch.empty(1, world * self.rows, dtype=torch.float16, device=dev)

    def describe(self):
        d = super().describe()
        d["workload"] = f"F1 RMSNorm -> GEMV, x [1,{self.d_in}] fp16, W [{self.d_ff},{self.d_in}] fp16"
        d["l2"] = (f"weights rotated over {self.nrep} replicas "
                   f"({self.nrep * self.rows * self.d_in * 2 / 1e6:.0f} MB per GPU)")
        return d

    def step_bytes_total(self):
        return self.costs.rmsnorm_gemv_bytes(1, self.d_in, self.d_ff)

    def launch_bytes(self):
        return self.costs.rmsnorm_gemv_bytes(1, self.d_in, self.rows)

    def torch_kernel(self, rep):
        """Library baseline: RMSNorm as PyTorch elementwise ops, then F.linear (cuBLAS)."""
        t = self.t
        xf = self.x.float()
        xn = (xf * t.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).half() * self.gamma
        return t.nn.functional.linear(xn, self.W[rep % self.nrep])

    def run_kernel(self, rep):
        W = self.W[rep % self.nrep]
        if self.fused():
            self.ops.rmsnorm_gemv(self.x, self.gamma, W, eps=1e-6, out=self.h_full, comm=self.comm)
        else:
            self.ops.rmsnorm_gemv(self.x, self.gamma, W, eps=1e-6, out=self.h_local)

    def e2e_step(self):
        W = self.W[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.x_dev, self.x_host)
        if self.world > 1 and self.comm is not None:
            h = self.ops.rmsnorm_gemv(self.x_dev, self.gamma, W, eps=1e-6, out=self.h_full,
                                      comm=self.comm)
        elif self.world == 1:
            self.ops.rmsnorm_gemv(self.x_dev, self.gamma, W, eps=1e-6,
                                  out=self.out_host.view(1, -1))
            return
        else:
            h = self.gather_rows(self.ops.rmsnorm_gemv(self.x_dev, self.gamma, W, eps=1e-6,
                                                       out=self.h_local))
        self.ops.stage(self.out_host, h.reshape(-1))

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.d_ff * frac_rows))
        self.cpu_rows = n
        self.cW = (rng.standard_normal((n, self.d_in), dtype=np.float32) / 64
                   ).astype(np.float16).astype(np.float32)
        self.cx = self.x_cpu.float().numpy()[0].copy()
        self.cg = self.g_cpu.float().numpy().copy()

    def cpu_step(self, threads):
        from oracle import oracle as O

        xn = O.rmsnorm_f32(self.cx, self.cg, 1e-6, use_ref=True)
        return O.ref_gemv_threaded(self.cW, xn, threads)

    def cpu_step_bytes(self):
        return self.costs.rmsnorm_gemv_bytes(1, self.d_in, self.cpu_rows)


class F4(Workload):
    """config C3: q [1,32,1,128]; K,V [1,32,4096,128] fp16, scale 1/sqrt(128).
    With N ranks the heads are sharded (32/N per rank), out all-gathered."""

    name = "f4"

    def __init__(self, rank, world, torch, H=32, L=4096, batch=1):
        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.H, self.L, self.batch = rank, world, H, L, batch
        self.h = H // world
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(7 + rank)
        per_rep = 2 * batch * self.h * L * 128 * 2
        self.nrep = min(64, max(2, math.ceil(2 * 126e6 / per_rep)))
        self.KV = [(torch.randn(batch, self.h, L, 128, generator=g, device=dev).half(),
                    torch.randn(batch, self.h, L, 128, generator=g, device=dev).half())
                   for _ in range(self.nrep)]
        xg = torch.Generator().manual_seed(42)
        self.q_cpu = torch.randn(batch, self.h, 128, generator=xg).half()
        self.q = self.q_cpu.to(dev)
        self.o = torch.empty_like(self.q)
        self.o_full = torch.empty(world, *self.o.shape, dtype=self.o.dtype, device=dev)

    def describe(self):
        return {"workload": f"F4 split-KV FlashDecode MHA, q [{self.batch},{self.H},1,128], "
                            f"K/V [{self.batch},{self.H},{self.L},128] fp16 (config C3)",
                "global_batch": self.batch, "heads": self.H, "kv_len": self.L,
                "parallelism": ("single GPU" if self.world == 1 else
                                f"heads sharded {self.h}/rank, {self.xname()} of out"),
                "kv_replicas": self.nrep,
                "l2": f"K/V rotated over {self.nrep} replicas"}

    def step_bytes_total(self):
        return self.costs.flashdecode_bytes([self.L] * self.batch, self.H, self.H)

    def launch_bytes(self):
        return self.costs.flashdecode_bytes([self.L] * self.batch, self.h, self.h)

    def run_kernel(self, rep):
        K, V = self.KV[rep % self.nrep]
        self.ops.flashdecode(self.q, K, V, out=self.o)

    def torch_kernel(self, rep):
        """Library baseline: torch scaled_dot_product_attention (its fused backends)."""
        K, V = self.KV[rep % self.nrep]
        q = self.q.unsqueeze(2)                      # [batch, H, 1, 128]
        return self.t.nn.functional.scaled_dot_product_attention(q, K, V)

    def exchange(self):
        if self.world > 1:
            self.gather_blocks(self.o, self.o_full)

    def e2e_setup(self):
        t = self.t
        self.q_host = self.q_cpu.pin_memory()
        self.out_host = t.empty(self.world * self.o.numel(), dtype=t.float16).pin_memory()
        self.q_dev = t.empty_like(self.q)
        self._e2e_i = 0
        return self.q_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        K, V = self.KV[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.q_dev, self.q_host)
        if self.world == 1:      # the kernel writes o straight into the pinned host buffer
            self.ops.flashdecode(self.q_dev, K, V, out=self.out_host.view_as(self.o))
            return
        o = self.gather_blocks(self.ops.flashdecode(self.q_dev, K, V, out=self.o))
        self.ops.stage(self.out_host, o.reshape(-1))

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.H * frac_rows))
        self.cpu_heads = n
        self.cq = rng.standard_normal((n, 128), dtype=np.float32) / math.sqrt(128)  # scale folded
        self.cK = rng.standard_normal((n, self.L, 128), dtype=np.float32)
        self.cV = rng.standard_normal((n, self.L, 128), dtype=np.float32)

    def cpu_step(self, threads):
        from oracle import oracle as O

        return O.attention_f32(self.cq, self.cK, self.cV, use_ref=True)

    def cpu_step_bytes(self):
        return self.costs.flashdecode_bytes([self.L], self.cpu_heads, self.cpu_heads)


class GQA(F4):
    """config C5: batch 8, 64 q heads, 8 kv heads, head_dim 128, bf16 paged
    KV (64-token pages, random page permutation), lengths ~U[1024, 32768] seeded.
    With N ranks the kv heads are sharded (8/N per rank with their 8 q heads)."""

    name = "gqa"

    def __init__(self, rank, world, torch, batch=8, hq=64, hkv=8, ps=64):
        import numpy as np

        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.batch = rank, world, batch
        self.hq_total, self.hkv_total = hq, hkv
        self.hkv, self.hq = hkv // world, hq // world
        rng = np.random.default_rng(2024)
        self.lens_np = rng.integers(1024, 32769, size=batch).astype(np.int32)
        pages_per = [(int(n) + ps - 1) // ps for n in self.lens_np]
        maxp = max(pages_per)
        npages = sum(pages_per)
        perm = rng.permutation(npages).astype(np.int32)
        table = np.zeros((batch, maxp), np.int32)
        o = 0
        for b, n in enumerate(pages_per):
            table[b, :n] = perm[o:o + n]
            o += n
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(11 + rank)
        kv_bytes = 2 * npages * self.hkv * ps * 128 * 2
        self.nrep = max(1, min(8, math.ceil(2 * 126e6 / kv_bytes)))
        self.KV = [(torch.randn(npages, self.hkv, ps, 128, generator=g, device=dev).bfloat16(),
                    torch.randn(npages, self.hkv, ps, 128, generator=g, device=dev).bfloat16())
                   for _ in range(self.nrep)]
        self.table = torch.from_numpy(table).to(dev)
        self.lens = torch.from_numpy(self.lens_np).to(dev)
        self.table_bytes = table.nbytes
        xg = torch.Generator().manual_seed(42)
        self.q_cpu = torch.randn(batch, self.hq, 128, generator=xg).bfloat16()
        self.q = self.q_cpu.to(dev)
        self.o = torch.empty_like(self.q)
        self.o_full = torch.empty(batch, hq, 128, dtype=self.o.dtype, device=dev)
        self.L = int(self.lens_np.max())
        self.H = hq

    def describe(self):
        return {"workload": "GQA paged FlashDecode, batch 8, 64 q / 8 kv heads, head_dim 128, "
                            "bf16, 64-token pages, lengths ~U[1024,32768] (config C5)",
                "global_batch": self.batch, "seq_lens": [int(x) for x in self.lens_np],
                "parallelism": ("single GPU" if self.world == 1 else
                                f"kv heads sharded {self.hkv}/rank, {self.xname()} of out"),
                "kv_replicas": self.nrep, "l2": f"paged K/V {self.nrep} replica(s), "
                f"{sum(t.nbytes for kv in self.KV for t in kv) / 1e6:.0f} MB > 126 MB L2"}

    def step_bytes_total(self):
        return self.costs.flashdecode_bytes(self.lens_np, self.hq_total, self.hkv_total,
                                            page_table_bytes=self.table_bytes)

    def launch_bytes(self):
        return self.costs.flashdecode_bytes(self.lens_np, self.hq, self.hkv,
                                            page_table_bytes=self.table_bytes)

    def run_kernel(self, rep):
        K, V = self.KV[rep % self.nrep]
        self.ops.flashdecode(self.q, K, V, seq_lens=self.lens, page_table=self.table, out=self.o)

    def exchange(self):
        # [batch, Hq / N, D] per rank -> [batch, Hq, D], heads in rank order
        if self.world > 1:
            self.gather_rows(self.o.view(self.batch, -1), self.o_full.view(self.batch, -1))

    def e2e_setup(self):
        t = self.t
        self.q_host = self.q_cpu.pin_memory()
        self.out_host = t.empty(self.world * self.o.numel(), dtype=t.bfloat16).pin_memory()
        self.q_dev = t.empty_like(self.q)
        self._e2e_i = 0
        return self.q_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        K, V = self.KV[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.q_dev, self.q_host)
        if self.world == 1:      # the kernel writes o straight into the pinned host buffer
            self.ops.flashdecode(self.q_dev, K, V, seq_lens=self.lens, page_table=self.table,
                                 out=self.out_host.view_as(self.o))
            return
        o = self.ops.flashdecode(self.q_dev, K, V, seq_lens=self.lens, page_table=self.table,
                                 out=self.o)
        o = self.gather_rows(o.view(self.batch, -1))
        self.ops.stage(self.out_host, o.reshape(-1))

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        L = max(64, int(int(self.lens_np[0]) * frac_rows))
        self.cpu_len = L
        # one sequence, one kv head with its 8 q heads, through the reference's attention_ref
        self.cq = rng.standard_normal((8, 128), dtype=np.float32) / math.sqrt(128)
        K = rng.standard_normal((L, 128), dtype=np.float32)
        V = rng.standard_normal((L, 128), dtype=np.float32)
        self.cK = np.broadcast_to(K, (8, L, 128)).copy()
        self.cV = np.broadcast_to(V, (8, L, 128)).copy()

    def cpu_step_bytes(self):
        return self.costs.flashdecode_bytes([self.cpu_len], 8, 1)


class MLP(Workload):
    """config C4: Llama-70B-shaped decode MLP, batch 16, d 8192, d_ff 28672,
    bf16; RMSNorm (eps 1e-5) -> gate/up -> SwiGLU -> down. With N ranks gate/up
    and down are column-sharded; h is all-gathered between them and y at the end."""

    name = "mlp"
    exchanges_per_step = 2
    kernels_per_step = 3   # prep, gate/up+SwiGLU, down (exchanges counted separately)

    def __init__(self, rank, world, torch, batch=16, d=8192, d_ff=28672):
        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.batch, self.d, self.d_ff = rank, world, batch, d, d_ff
        self.ff, self.dd = d_ff // world, d // world
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(70 + rank)
        self.nrep = 1   # 1.41 GB / N per replica, > L2 for N <= 8
        self.Wg = (torch.randn(self.ff, d, generator=g, device=dev) / math.sqrt(d)).bfloat16()
        self.Wu = (torch.randn(self.ff, d, generator=g, device=dev) / math.sqrt(d)).bfloat16()
        self.Wd = (torch.randn(self.dd, d_ff, generator=g, device=dev) / math.sqrt(d_ff)).bfloat16()
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(batch, d, generator=xg).bfloat16()
        self.x = self.x_cpu.to(dev)
        self.gamma = torch.ones(d, dtype=torch.bfloat16, device=dev)
        self.h = torch.empty(batch, self.ff, dtype=torch.bfloat16, device=dev)
        self.h_full = torch.empty(batch, d_ff, dtype=torch.bfloat16, device=dev)
        self.y = torch.empty(batch, self.dd, dtype=torch.bfloat16, device=dev)
        self.y_full = torch.empty(batch, d, dtype=torch.bfloat16, device=dev)

    def describe(self):
        return {"workload": "Llama-70B-shaped decode MLP, batch 16, d 8192, d_ff 28672, bf16: "
                            "RMSNorm -> gate/up -> SwiGLU -> down (config C4)",
                "global_batch": self.batch, "d_model": self.d, "d_ff": self.d_ff,
                "parallelism": ("single GPU" if self.world == 1 else
                                f"tp{self.world}: gate/up and down column-sharded, "
                                f"{self.xname()} of h and of y"),
                "l2": "weights 1.41 GB / N per GPU, read once per step (> 126 MB L2)"}

    def step_bytes_total(self):
        return self.costs.mlp_bytes(self.batch, self.d, self.d_ff)

    def launch_bytes(self):
        return self.costs.mlp_bytes(self.batch, self.d, self.d_ff) // self.world

    def _gather_h(self):
        if self.world == 1:
            return self.h
        if not self.with_exchange:     # kernel-only timing: the down GEMV reads h_full as is
            return self.h_full
        return self.gather_rows(self.h, self.h_full)

    def run_kernel(self, rep):
        self.ops.gateup_swiglu(self.x, self.Wg, self.Wu, gamma=self.gamma, eps=1e-5, out=self.h)
        self.ops.gemv(self._gather_h(), self.Wd, out=self.y)

    def torch_kernel(self, rep):
        """Library baseline: RMSNorm, gate/up, SwiGLU and down with PyTorch ops (cuBLAS)."""
        t, F = self.t, self.t.nn.functional
        xf = self.x.float()
        xn = (xf * t.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).bfloat16() * self.gamma
        return F.linear(F.silu(F.linear(xn, self.Wg)) * F.linear(xn, self.Wu), self.Wd)

    def exchange(self):
        if self.world > 1:
            self.gather_rows(self.y, self.y_full)

    def e2e_setup(self):
        t = self.t
        self.x_host = self.x_cpu.pin_memory()
        self.out_host = t.empty(self.world * self.y.numel(), dtype=t.bfloat16).pin_memory()
        self.x_dev = t.empty_like(self.x)
        return self.x_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        self.ops.stage(self.x_dev, self.x_host)
        h = self.ops.gateup_swiglu(self.x_dev, self.Wg, self.Wu, gamma=self.gamma, eps=1e-5,
                                   out=self.h)
        if self.world > 1:
            h = self.gather_rows(h)
        # (the tcgen05 epilogue writes 32-byte pieces across batch rows: slow into host
        # memory, so the result goes out by one staging copy instead)
        y = self.ops.gemv(h, self.Wd, out=self.y)
        if self.world > 1:
            y = self.gather_rows(y)
        self.ops.stage(self.out_host, y.reshape(-1))

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.d_ff * frac_rows))
        self.cpu_rows = n
        self.cWg = rng.standard_normal((n, self.d), dtype=np.float32) / math.sqrt(self.d)
        self.cWu = rng.standard_normal((n, self.d), dtype=np.float32) / math.sqrt(self.d)
        self.cx = self.x_cpu.float().numpy()

    def cpu_step(self, threads):
        import numpy as np

        from oracle import oracle as O

        for b in range(self.batch):
            xn = O.rmsnorm_f32(self.cx[b], np.ones(self.d, np.float32), 1e-5, use_ref=True)
            O.swiglu_f32(O.ref_gemv_threaded(self.cWg, xn, threads),
                         O.ref_gemv_threaded(self.cWu, xn, threads), use_ref=True)

    def cpu_step_bytes(self):
        return 2 * (2 * self.cpu_rows * self.d)


class F2FP8(F2):
    """F2 (config C2's shape) with e4m3 weights and per-row fp32 scales: the weight
    stream is half of C2's bytes (scope's next rows: low-precision weight formats;
    not one of the five benchmark configs). Single GPU."""

    name = "f2fp8"

    def __init__(self, rank, world, torch, d_in=4096, d_ff=11008, batch=1):
        if world > 1:
            raise SystemExit("the f2fp8 workload runs on one GPU")
        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world = rank, world
        self.d_in, self.d_ff, self.batch, self.rows = d_in, d_ff, batch, d_ff
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(1234)
        sc = 1.0 / math.sqrt(d_in)
        per_rep = 2 * d_ff * d_in
        self.nrep = min(64, max(2, math.ceil(2 * 126e6 / per_rep)))
        self.W = []
        for _ in range(self.nrep):
            Wg8, sg = ops.quantize_fp8_rows(torch.randn(d_ff, d_in, generator=g, device=dev) * sc)
            Wu8, su = ops.quantize_fp8_rows(torch.randn(d_ff, d_in, generator=g, device=dev) * sc)
            self.W.append((Wg8, sg, Wu8, su))
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(batch, d_in, generator=xg).half()
        self.x = self.x_cpu.to(dev)
        self.h_local = torch.empty(batch, d_ff, dtype=torch.float16, device=dev)
        self.h_full = self.h_local

    def describe(self):
        return {"workload": f"F2 gate+up GEMV -> SwiGLU with e4m3 weights + per-row fp32 scales, "
                            f"x [{self.batch},{self.d_in}] fp16, Wg/Wu [{self.d_ff},{self.d_in}] fp8",
                "global_batch": self.batch, "d_in": self.d_in, "d_ff": self.d_ff,
                "parallelism": "single GPU", "weight_replicas": self.nrep,
                "l2": f"weights rotated over {self.nrep} replicas "
                      f"({self.nrep * 2 * self.d_ff * self.d_in / 1e6:.0f} MB > 126 MB L2)"}

    def _bytes(self):
        return 2 * self.d_ff * self.d_in + 2 * self.d_ff * 4 + self.batch * (self.d_in + self.d_ff) * 2

    def step_bytes_total(self):
        return self._bytes()

    def launch_bytes(self):
        return self._bytes()

    def run_kernel(self, rep):
        Wg8, sg, Wu8, su = self.W[rep % self.nrep]
        self.ops.gateup_swiglu_fp8(self.x, Wg8, sg, Wu8, su, out=self.h_local)

    def exchange(self):
        pass

    def e2e_step(self):
        Wg8, sg, Wu8, su = self.W[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.x_dev, self.x_host)
        h = self.ops.gateup_swiglu_fp8(self.x_dev, Wg8, sg, Wu8, su, out=self.h_local)
        self.ops.stage(self.out_host, h.reshape(-1))


class QKV(Workload):
    """The step before FlashDecode (next row of the scope, not one of the five benchmark configs):
    RMSNorm -> QKV projection -> RoPE -> KV-cache append, Llama-3-8B shapes:
    x [1, 4096] fp16, Wqkv [(32 + 2 x 8) x 128, 4096], paged cache (64-token pages).
    With N ranks each owns Hq/N query and Hkv/N kv heads (the attention that
    follows is sharded the same way), so no exchange is needed."""

    name = "qkv"
    exchanges_per_step = 0

    def __init__(self, rank, world, torch, d=4096, hq=32, hkv=8, D=128, ps=64):
        import numpy as np

        from decodebench_b200 import costs, ops

        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.batch, self.d_in = rank, world, 1, d
        if hkv % world:
            raise SystemExit(f"{hkv} kv heads do not split over {world} ranks")
        self.hq_total, self.hkv_total, self.D = hq, hkv, D
        self.hq, self.hkv = hq // world, hkv // world
        self.rows = (self.hq + 2 * self.hkv) * D
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(31 + rank)
        per_rep = self.rows * d * 2
        self.nrep = min(64, max(2, math.ceil(2 * 126e6 / per_rep)))
        self.W = [ops.interleave_rope_rows(
            (torch.randn(self.rows, d, generator=g, device=dev) / 64).half(), self.hq, self.hkv, D)
            for _ in range(self.nrep)]
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(1, d, generator=xg).half()
        self.g_cpu = torch.randn(d, generator=xg).half()
        self.x, self.gamma = self.x_cpu.to(dev), self.g_cpu.to(dev)
        self.inv_freq = ops.rope_inv_freq(D, 500000.0, device=dev)
        self.max_pages = 128
        self.pos = torch.tensor([self.max_pages * ps - 1000], dtype=torch.int32, device=dev)
        self.table = torch.from_numpy(np.arange(self.max_pages, dtype=np.int32)[None, :]).to(dev)
        self.kc = torch.zeros(self.max_pages, self.hkv, ps, D, dtype=torch.float16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        self.q = torch.empty(1, self.hq, D, dtype=torch.float16, device=dev)

    def describe(self):
        return {"workload": "QKV projection + RoPE + paged KV append (the step before FlashDecode), "
                            f"x [1,{self.d_in}] fp16, Wqkv [{(self.hq_total + 2 * self.hkv_total) * self.D},"
                            f"{self.d_in}] fp16, 32 q / 8 kv heads, head_dim 128",
                "global_batch": 1, "d_in": self.d_in,
                "parallelism": ("single GPU" if self.world == 1 else
                                f"heads sharded ({self.hq} q / {self.hkv} kv per rank), no exchange"),
                "weight_replicas": self.nrep,
                "l2": f"weights rotated over {self.nrep} replicas "
                      f"({self.nrep * self.rows * self.d_in * 2 / 1e6:.0f} MB per GPU > 126 MB L2)"}

    def _bytes(self, rows, hq, hkv):
        return rows * self.d_in * 2 + 2 * self.d_in * 2 + hq * self.D * 2 + 2 * hkv * self.D * 2

    def step_bytes_total(self):
        return self._bytes((self.hq_total + 2 * self.hkv_total) * self.D, self.hq_total, self.hkv_total)

    def launch_bytes(self):
        return self._bytes(self.rows, self.hq, self.hkv)

    def run_kernel(self, rep):
        self.ops.qkv_rope_append(self.x, self.W[rep % self.nrep], self.pos, self.inv_freq,
                                 self.kc, self.vc, self.hq, self.hkv, page_table=self.table,
                                 gamma=self.gamma, out=self.q)

    def exchange(self):
        pass

    def e2e_setup(self):
        t = self.t
        self.x_host = self.x_cpu.pin_memory()
        self.out_host = t.empty(self.q.numel(), dtype=t.float16).pin_memory()
        self.x_dev = t.empty_like(self.x)
        self._e2e_i = 0
        return self.x_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        W = self.W[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.x_dev, self.x_host)
        q = self.ops.qkv_rope_append(self.x_dev, W, self.pos, self.inv_freq, self.kc, self.vc,
                                     self.hq, self.hkv, page_table=self.table, gamma=self.gamma,
                                     out=self.q)
        self.ops.stage(self.out_host, q.reshape(-1))

    # CPU: the reference's gemv_ref over a sample of the weight rows (the projection
    # is the whole cost of the step)
    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.rows * frac_rows))
        self.cpu_rows = n
        self.cW = (rng.standard_normal((n, self.d_in), dtype=np.float32) / 64
                   ).astype(np.float16).astype(np.float32)
        self.cx = self.x_cpu.float().numpy()[0].copy()

    def cpu_step(self, threads):
        from oracle import oracle as O

        return O.ref_gemv_threaded(self.cW, self.cx, threads)

    def cpu_step_bytes(self):
        return self.cpu_rows * self.d_in * 2


class Layer(Workload):
    """One whole Llama decode layer for one new token (the scope's next rows, not a
    benchmark config): d 4096, 32 q / 8 kv heads, FFN 11008, fp16, contiguous cache
    of 1024 tokens + the new one; four kernels chained with programmatic dependent
    launch (QKV + RoPE + append, FlashDecode, o_proj + residual, and the persistent
    MLP block: RMSNorm + gate/up + SwiGLU, grid barrier, down + residual). Single GPU: a sharded layer needs a reduction after
    o_proj and down, which this build does not provide."""

    name = "layer"
    kernels_per_step = 5
    exchanges_per_step = 0

    def __init__(self, rank, world, torch):
        if world > 1:
            raise SystemExit("the layer workload runs on one GPU")
        from decodebench_b200.demos.llama_decode import build_demo

        self.t = torch
        self.rank, self.world, self.batch = rank, world, 1
        _, self.inputs, self.reps, self.fused = build_demo("layer", dim=4096, batch=1)
        self.nrep = len(self.reps)
        self.out = None
        from decodebench_b200 import ops

        # the MLP block is one persistent launch unless DBK_MLP_BLOCK=0 (o_proj joins it
        # with DBK_LAYER_TAIL=1)
        self.fused(self.reps[0])
        if ops._MLP_BLOCK and not ops._mlp_block_refused:
            self.kernels_per_step = 3 if ops._LAYER_TAIL else 4

    def describe(self):
        return {"workload": "whole Llama decode layer, d 4096, 32 q / 8 kv heads, FFN 11008, fp16, "
                            "1024 cached tokens + 1 new", "global_batch": 1,
                "parallelism": "single GPU", "weight_replicas": self.nrep,
                "l2": f"weights rotated over {self.nrep} replicas (> 126 MB L2 each)"}

    def step_bytes_total(self):
        inp = self.inputs
        w = sum(inp[k].nbytes for k in ("Wqkv_il", "Wo", "Wg", "Wu", "Wd"))
        _, hkv, _, dh = inp["Kc"].shape
        kv = 2 * (1024 + 1) * hkv * dh * 2
        return w + kv + 2 * inp["x"].nbytes

    def launch_bytes(self):
        return self.step_bytes_total()

    def run_kernel(self, rep):
        self.out = self.fused(self.reps[rep % self.nrep])

    def exchange(self):
        pass

    def e2e_setup(self):
        t = self.t
        self.x_host = self.inputs["x"].cpu().pin_memory()
        self.out_host = t.empty(self.inputs["x"].numel(), dtype=t.float16).pin_memory()
        self._e2e_i = 0
        return self.x_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        from decodebench_b200 import ops

        r = self.reps[self._e2e_i % self.nrep]
        self._e2e_i += 1
        ops.stage(r["x"], self.x_host)
        y = self.fused(r)
        ops.stage(self.out_host, y.reshape(-1))

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        rows = 6144 + 4096 + 2 * 11008
        n = max(1, int(rows * frac_rows))
        self.cpu_rows = n
        self.cW = (rng.standard_normal((n, 4096), dtype=np.float32) / 64).astype(np.float16).astype(np.float32)
        self.cx = self.inputs["x"].float().cpu().numpy()[0].copy()

    def cpu_step(self, threads):
        from oracle import oracle as O

        return O.ref_gemv_threaded(self.cW, self.cx, threads)

    def cpu_step_bytes(self):
        return self.cpu_rows * 4096 * 2


class MLPBlock(Workload):
    """The decode MLP block at batch 1 in one persistent launch (dbk_mlp_block):
    RMSNorm -> gate/up [11008, 4096] -> SwiGLU -> grid barrier -> down [4096, 11008]
    + residual, fp16 (C2's F2 followed by its down projection; the scope's next
    rows, not a benchmark config). Single GPU."""

    name = "mlpblock"
    exchanges_per_step = 0

    def __init__(self, rank, world, torch, d=4096, d_ff=11008, batch=1):
        from decodebench_b200 import costs, ops

        if world > 1:
            raise SystemExit("the mlpblock workload runs on one GPU")
        self.t, self.ops, self.costs = torch, ops, costs
        self.rank, self.world, self.batch, self.d, self.d_ff = rank, world, batch, d, d_ff
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(77)
        per_rep = 3 * d * d_ff * 2
        self.nrep = max(2, math.ceil(2 * 126e6 / per_rep))

        def w(r, c):
            return (torch.randn(r, c, generator=g, device=dev) / math.sqrt(c)).half()
        self.W = [(w(d_ff, d), w(d_ff, d), w(d, d_ff)) for _ in range(self.nrep)]
        xg = torch.Generator().manual_seed(42)
        self.x_cpu = torch.randn(batch, d, generator=xg).half()
        self.x = self.x_cpu.to(dev)
        self.gamma = (1 + 0.1 * torch.randn(d, generator=xg)).half().to(dev)
        self.h = torch.empty(batch, d_ff, dtype=torch.float16, device=dev)
        self.y = torch.empty(batch, d, dtype=torch.float16, device=dev)

    def describe(self):
        return {"workload": f"decode MLP block in one persistent launch: RMSNorm -> gate/up "
                            f"[{self.d_ff},{self.d}] -> SwiGLU -> down [{self.d},{self.d_ff}] + "
                            f"residual, x [{self.batch},{self.d}] fp16",
                "global_batch": self.batch, "d_model": self.d, "d_ff": self.d_ff,
                "parallelism": "single GPU", "weight_replicas": self.nrep,
                "l2": f"weights rotated over {self.nrep} replicas "
                      f"({self.nrep * 3 * self.d * self.d_ff * 2 / 1e6:.0f} MB > 126 MB L2)"}

    def step_bytes_total(self):
        # three weight matrices, x, gamma, y and the residual read (h stays on chip / in L2)
        return self.costs.mlp_bytes(self.batch, self.d, self.d_ff) + 2 * self.batch * self.d

    def launch_bytes(self):
        return self.step_bytes_total()

    def run_kernel(self, rep):
        Wg, Wu, Wd = self.W[rep % self.nrep]
        self.ops.mlp_block(self.x, Wg, Wu, Wd, gamma=self.gamma, eps=1e-5, residual=self.x,
                           out=self.y, h=self.h)

    def exchange(self):
        pass

    def torch_kernel(self, rep):
        """Library baseline: the same block with PyTorch ops (cuBLAS GEMVs)."""
        F = self.t.nn.functional
        Wg, Wu, Wd = self.W[rep % self.nrep]
        a = F.rms_norm(self.x, (self.d,), self.gamma, 1e-5)
        return F.linear(F.silu(F.linear(a, Wg)) * F.linear(a, Wu), Wd) + self.x

    def e2e_setup(self):
        t = self.t
        self.x_host = self.x_cpu.pin_memory()
        self.out_host = t.empty(self.batch * self.d, dtype=t.float16).pin_memory()
        self.x_dev = t.empty_like(self.x)
        self._e2e_i = 0
        return self.x_host.nbytes, self.out_host.nbytes

    def e2e_step(self):
        Wg, Wu, Wd = self.W[self._e2e_i % self.nrep]
        self._e2e_i += 1
        self.ops.stage(self.x_dev, self.x_host)
        self.ops.mlp_block(self.x_dev, Wg, Wu, Wd, gamma=self.gamma, eps=1e-5,
                           residual=self.x_dev, out=self.out_host.view(self.batch, -1), h=self.h)

    def cpu_setup(self, frac_rows: float = 1.0):
        import numpy as np

        rng = np.random.default_rng(5)
        n = max(1, int(self.d_ff * frac_rows))
        self.cpu_rows = n
        mk = lambda r, c: (rng.standard_normal((r, c), dtype=np.float32) / math.sqrt(c)  # noqa: E731
                           ).astype(np.float16).astype(np.float32)
        self.cWg, self.cWu = mk(n, self.d), mk(n, self.d)
        self.cWd = mk(max(1, int(self.d * frac_rows)), n)
        self.cx = self.x_cpu.float().numpy()[0].copy()

    def cpu_step(self, threads):
        from oracle import oracle as O

        g = O.ref_gemv_threaded(self.cWg, self.cx, threads)
        u = O.ref_gemv_threaded(self.cWu, self.cx, threads)
        h = O.swiglu_f32(g, u, use_ref=True)
        return O.ref_gemv_threaded(self.cWd, h, threads)

    def cpu_step_bytes(self):
        return 2 * (2 * self.cpu_rows * self.d + self.cWd.size)


WORKLOADS = {"f2": F2, "f1": F1, "f4": F4, "gqa": GQA, "mlp": MLP, "qkv": QKV, "layer": Layer,
             "f2fp8": F2FP8, "mlpblock": MLPBlock}


# ---------------------------------------------------------------- timing
def dist_max(torch, v: float) -> float:
    if not torch.distributed.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier_sync(torch):
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.cuda.synchronize()


def _capture(torch, body):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    return g


class StepGraphs:
    """CUDA graphs of the step. `prepare(n)` captures one graph of exactly n
    consecutive steps (rotating the weight replicas; consecutive kernels overlap
    prologue and tail through programmatic dependent launch), and `run(n)`
    replays it, so a timed region of K steps is one graph launch whatever K is.
    Counts above `cap` replay a cap-step graph several times."""

    def __init__(self, torch, wl, with_exchange: bool, cap: int = 4096):
        self.torch = torch
        self.wl = wl
        self.cap = cap
        self.graphs = {}

        def one(r):
            wl.with_exchange = with_exchange
            wl.run_kernel(r)
            if with_exchange:
                wl.exchange()
        self.one = one

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):          # warm-up outside capture (workspaces, attributes)
            for r in range(wl.nrep):
                one(r)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()

    def _chunks(self, steps: int) -> list[int]:
        out = [self.cap] * (steps // self.cap)
        if steps % self.cap:
            out.append(steps % self.cap)
        return out

    def prepare(self, *counts: int) -> None:
        for steps in counts:
            for n in self._chunks(steps):
                if n not in self.graphs:
                    self.graphs[n] = _capture(
                        self.torch, lambda n=n: [self.one(r % self.wl.nrep) for r in range(n)])
        self.torch.cuda.synchronize()

    def run(self, steps: int) -> None:
        for n in self._chunks(steps):
            if n not in self.graphs:
                raise RuntimeError(f"no graph of {n} steps captured (call prepare({n}) first)")
            self.graphs[n].replay()


_FLUSH = {}


def l2_flush(torch) -> None:
    """Overwrite a 256 MB buffer (twice the 126 MB L2) on the current device."""
    dev = torch.cuda.current_device()
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = _FLUSH[dev] = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    buf.zero_()


def timed(torch, run, steps: int, warmup: int, host_latency: bool = True) -> float:
    """Device ms for run(steps) after run(warmup); barrier + sync on both sides,
    CUDA events on the current stream, max over ranks.

    With host_latency=False, L2 is flushed (the warm-up's last replicas would
    otherwise still be cached for the first timed steps) and a short device-side
    delay is queued ahead of the start event, so the work that run() submits is
    already queued when the start event fires: the region times the steps on the
    device, not the host's submission of a graph (several us per replay, which
    would otherwise weigh on short runs)."""
    if warmup:
        run(warmup)
    barrier_sync(torch)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    if not host_latency:
        l2_flush(torch)
        torch.cuda._sleep(DELAY_CYCLES)
    a.record()
    run(steps)
    b.record()
    barrier_sync(torch)
    return dist_max(torch, a.elapsed_time(b))


def loop(fn):
    def run(n):
        for _ in range(n):
            fn()
    return run


def cpu_time(wl, threads: int, budget_s: float, steps: int | None = None, warmup: int = 1,
             min_steps: int = 10):
    """Median seconds per CPU step; steps=None -> as many as fit in budget_s (at
    least min_steps)."""
    # Warm up for at least `warmup` steps and ~1.5 s, so thread pools, page
    # faults and CPU clock ramp are behind the measured steps.
    t_warm = time.perf_counter() + 1.5
    n_warm = 0
    while n_warm < warmup or time.perf_counter() < t_warm:
        wl.cpu_step(threads)
        n_warm += 1
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        wl.cpu_step(threads)
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() >= t_end and len(times) >= min_steps:
            break
    return statistics.median(times), len(times)


def cpu_baseline(wl, threads: int, budget_s: float, steps=None, warmup=1) -> dict:
    # Size the sample so one step takes <= ~budget/5 s.
    wl.cpu_setup(1.0)
    t0 = time.perf_counter()
    wl.cpu_step(threads)
    one = time.perf_counter() - t0
    frac = 1.0
    if steps is not None and one * (steps + warmup) > budget_s:
        frac = max(budget_s / ((steps + warmup) * one), 1e-3)
        wl.cpu_setup(frac)
    med, n = cpu_time(wl, threads, budget_s, steps=steps, warmup=warmup)
    gbs = wl.cpu_step_bytes() / med / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "us_per_step": round(med * 1e6, 1),
            "sample": (f"{n} steps of the reference's own cpu_reference.cpp "
                       f"(oracle/_ref, gemv_ref rows split over {threads} threads) on "
                       f"{'the full step' if frac >= 1 else f'{frac:.3f} of the rows'}; "
                       "weights pre-converted fp16->fp32 once, untimed; median step time, "
                       "GB/s over the same algorithmic fp16 bytes")}


# Device-side delay (GPU clock cycles, ~100 us) queued ahead of a device-timed region.
DELAY_CYCLES = 200_000

# Seconds of CPU work per cpu_baseline measurement (both arms).
CPU_BUDGET_S = 12.0


# ---------------------------------------------------------------- main
def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference", "torch"], default="ours",
                    help="ours: this build's kernels; reference: the reference's CPU "
                         "implementation; torch: the same step with PyTorch / cuBLAS ops "
                         "(a library baseline, one GPU)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="f2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="f1/f2 only: output rows instead of the config's (e.g. 14336, the "
                         "shape of the reference's own published F1/F2 timings)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()

    if args.impl == "reference":
        if rank != 0:
            return 0
        sys.path.insert(0, str(ROOT))
        from oracle import oracle as O

        if not O.have_ref():
            print(json.dumps({"impl": "reference", "unavailable":
                              "oracle/_ref/libdbref.so (the reference's cpu_reference.cpp) not built"}))
            return 0
        torch.set_num_threads(threads)
        wl = WORKLOADS[args.workload].__new__(WORKLOADS[args.workload])
        _cpu_only_init(wl, args.workload, torch)
        # The same sampler, budget and warm-up as the GPU arm's cpu_baseline leg, so
        # the two CPU numbers describe the same measurement.
        cb = cpu_baseline(wl, threads, budget_s=CPU_BUDGET_S)
        us = cb["us_per_step"]
        line = {"metric": METRIC, "value": cb["value"], "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(us / 1e3, 4), "us_per_step": us, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (CPU reference on fp16 data)",
                "data": "synthetic, seeded", "config": wl.describe_cpu(),
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    if args.impl == "torch":
        return torch_arm(args, torch, world, rank)

    if world > 1:
        torch.cuda.set_device(local)
        import datetime

        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local),
                                             timeout=datetime.timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    dev_index = torch.cuda.current_device()

    sys.path.insert(0, str(ROOT))
    if args.rows and args.workload == "f2":
        wl = F2(rank, world, torch, d_ff=args.rows)
    elif args.rows and args.workload == "f1":
        wl = F1(rank, world, torch, d_out=args.rows)
    else:
        wl = WORKLOADS[args.workload](rank, world, torch)
    if world > 1 and os.environ.get("DBK_EXCHANGE", "peer") != "nccl":
        from decodebench_b200.comm import PeerComm

        wl.comm = PeerComm(8 << 20)       # largest block here: MLP h, 16 x 14336 bf16 at N=2

    # --- device-timed value: graphs of kernel + exchange, rotated over replicas
    graphs = StepGraphs(torch, wl, with_exchange=True)
    graphs.prepare(args.warmup, args.steps, 256)
    sampler = ClockSampler(dev_index)
    sampler.start()
    graphs.run(args.warmup)
    barrier_sync(torch)
    t_begin = time.perf_counter()
    ms = timed(torch, graphs.run, args.steps, 0, host_latency=False)
    t_end = time.perf_counter()
    # Keep identical steps running until the sampler has seen >= 5 samples, so
    # that a short timed region still has a clock record around it.
    # The graphs hold collectives, so every rank must replay the same number of
    # times: the decision to pad once more is agreed (max over ranks) each round.
    pad_until = time.perf_counter() + 2.0
    while True:
        need = (sampler.ok and sampler.count_between(t_begin, time.perf_counter()) < 5
                and time.perf_counter() < pad_until)
        if dist_max(torch, float(need)) == 0.0:
            break
        graphs.run(256)
        torch.cuda.synchronize()
    clocks = sampler.summary(t_begin, max(t_end, time.perf_counter()))
    sampler.stop()
    us_step = ms * 1e3 / args.steps
    value = wl.step_bytes_total() / (us_step * 1e-6) / 1e9

    # --- kernel-only timing for the roofline (the dominant, and only, kernel)
    if world > 1:
        kgraphs = StepGraphs(torch, wl, with_exchange=False)
        kgraphs.prepare(args.warmup, args.steps)
        kms = timed(torch, kgraphs.run, args.steps, args.warmup, host_latency=False)
    else:
        kms = ms
    k_us = kms * 1e3 / args.steps
    peak, peak_src = peaks()
    achieved = wl.launch_bytes() / (k_us * 1e-6) / 1e9
    tr = traffic_table().get(f"{wl.name}@{world}")
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": tr,
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                else "fallback 6650 GB/s", "kernel_us": round(k_us, 3),
                "bytes_per_launch": wl.launch_bytes()}

    # --- e2e through the public API with host buffers. Every step stages its input
    # in from pinned host memory and its result out to pinned host memory. Timed
    # twice: eagerly (one Python call per op, as a script calls the ops) and as
    # one CUDA graph of the same K steps (as a decode engine drives them).
    h2d, d2h = wl.e2e_setup()
    host = {}

    def e2e_run(n):
        t0 = time.perf_counter()
        for _ in range(n):
            wl.e2e_step()
        host["us"] = (time.perf_counter() - t0) * 1e6 / max(n, 1)
    eager_ms = timed(torch, e2e_run, args.steps, args.warmup)
    eager_us = eager_ms * 1e3 / args.steps
    egraphs = {}
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_cap):
        wl.e2e_step()
    torch.cuda.current_stream().wait_stream(s_cap)
    for n in {args.warmup, args.steps}:
        egraphs[n] = _capture(torch, lambda n=n: [wl.e2e_step() for _ in range(n)])
    torch.cuda.synchronize()
    egraphs[args.warmup].replay()
    e_ms = timed(torch, lambda n: egraphs[n].replay(), args.steps, 0, host_latency=False)
    e_us = e_ms * 1e3 / args.steps
    e2e = {"value": round(wl.step_bytes_total() / (e_us * 1e-6) / 1e9, 1), "unit": "GB/s",
           "us_per_step": round(e_us, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "mode": "one CUDA graph of the K steps, each step: H2D input, op, D2H result",
           "eager_us_per_step": round(eager_us, 3),
           "eager_value": round(wl.step_bytes_total() / (eager_us * 1e-6) / 1e9, 1),
           "host_enqueue_us_per_step": round(host.get("us", 0.0), 3),
           "path": "decodebench_b200.ops (ctypes -> libdbk.so C ABI); input in by ops.stage (dbk_copy: a kernel reading the pinned host buffer); at N=1 the batch<=8 ops and FlashDecode write their result straight into a pinned host buffer (out=); otherwise (the MLP's tcgen05 path, N>1) the result goes out by ops.stage"}

    line = None
    if rank == 0:
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as O

            if O.have_ref():
                torch.set_num_threads(threads)
                cb = cpu_baseline(wl, threads, budget_s=CPU_BUDGET_S)
        line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us_step / 1e3, 6),
                "us_per_step": round(us_step, 3), "hbm_frac_of_peak": round(value / world / peak, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "fp16", "data": "synthetic, seeded (torch.Generator)",
                "config": wl.describe(), "roofline": roofline, "cpu_baseline": cb, "e2e": e2e,
                "timing": ("one CUDA graph of exactly the K timed steps, replayed once between "
                           "two CUDA events on the launching stream; L2 is flushed (256 MB write) "
                           "and a ~100 us device-side delay is queued first, so the timed steps "
                           "start from a cold L2 with the graph already queued (host submission "
                           "latency excluded); weights rotate over replicas > 2x L2; max over ranks"),
                "clocks": clocks, "gpu_launches": args.steps * (wl.kernels_per_step + (
                    wl.exchanges_per_step if world > 1 and wl.comm is not None else 0))}
        print(json.dumps(line))
    if world > 1:
        # Every collective has completed (the e2e timing ended with a barrier and a
        # max-reduce). The step graphs still hold NCCL work, and tearing the
        # communicator down under them can block, so the ranks leave directly.
        torch.distributed.barrier()
        torch.cuda.synchronize()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)
    return 0


def torch_arm(args, torch, world, rank) -> int:
    """The workload's step computed with PyTorch library ops (cuBLAS GEMV, SDPA) on
    the same replicas, replayed from one CUDA graph of K steps: the library
    baseline printed beside this build's numbers."""
    if world > 1:
        if rank == 0:
            print(json.dumps({"impl": "torch", "unavailable": "the library arm runs on one GPU"}))
        return 0
    torch.cuda.set_device(0)
    sys.path.insert(0, str(ROOT))
    if args.rows and args.workload == "f2":
        wl = F2(0, 1, torch, d_ff=args.rows)
    elif args.rows and args.workload == "f1":
        wl = F1(0, 1, torch, d_out=args.rows)
    else:
        wl = WORKLOADS[args.workload](0, 1, torch)
    if not hasattr(wl, "torch_kernel"):
        print(json.dumps({"impl": "torch", "unavailable":
                          f"no PyTorch library path for workload {args.workload}"}))
        return 0
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_cap):
        for r in range(wl.nrep):
            wl.torch_kernel(r)
    torch.cuda.current_stream().wait_stream(s_cap)
    graphs = {}
    for n in {args.warmup, args.steps}:
        graphs[n] = _capture(torch, lambda n=n: [wl.torch_kernel(r % wl.nrep) for r in range(n)])
    graphs[args.warmup].replay()
    ms = timed(torch, lambda n: graphs[n].replay(), args.steps, 0, host_latency=False)
    us = ms * 1e3 / args.steps
    peak, _ = peaks()
    gbs = wl.step_bytes_total() / (us * 1e-6) / 1e9
    print(json.dumps({"metric": METRIC, "impl": "torch", "value": round(gbs, 1), "unit": "GB/s",
                      "us_per_step": round(us, 3), "frac_of_hbm_peak": round(gbs / peak, 4),
                      "steps": args.steps, "warmup": args.warmup, "config": wl.describe(),
                      "path": "torch ops on the same replicas (F.linear -> cuBLAS GEMV; "
                              "scaled_dot_product_attention), one CUDA graph of K steps"}))
    return 0


def _cpu_only_init(wl, name, torch):
    """Set up a workload for the CPU reference arm without touching a GPU."""
    from decodebench_b200 import costs

    wl.costs = costs
    gen = torch.Generator().manual_seed(42)
    if name in ("f2", "f1"):
        wl.batch, wl.d_in = 1, 4096
        wl.d_ff = 11008 if name == "f2" else 4096
        wl.x_cpu = torch.randn(1, wl.d_in, generator=gen).half()
        wl.g_cpu = torch.randn(wl.d_in, generator=gen).half()
        label = ("F2 gate+up GEMV -> SwiGLU, x [1,4096] fp16, Wg/Wu [11008,4096] (config C2)"
                 if name == "f2" else "F1 RMSNorm -> GEMV, x [1,4096], W [4096,4096]")
        wl.describe_cpu = lambda: {"workload": label, "global_batch": 1, "d_in": 4096,
                                   "d_ff": wl.d_ff, "parallelism": "CPU host threads"}
    elif name == "mlpblock":
        wl.batch, wl.d, wl.d_ff = 1, 4096, 11008
        wl.x_cpu = torch.randn(1, wl.d, generator=gen).half()
        wl.describe_cpu = lambda: {"workload": "decode MLP block: gate/up [11008,4096] -> SwiGLU "
                                               "-> down [4096,11008], x [1,4096] fp16",
                                   "global_batch": 1, "parallelism": "CPU host threads"}
    else:
        wl.H, wl.L, wl.batch = 32, 4096, 1
        wl.describe_cpu = lambda: {"workload": "F4 MHA q [1,32,1,128], K/V [1,32,4096,128]",
                                   "global_batch": 1, "parallelism": "CPU"}


if __name__ == "__main__":
    sys.exit(main())
