"""Benchmark of the hexkernels hot path on B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl ours|reference] [--ops all|none]

Workloads (the benchmark configurations, synthetic seeded inputs, all inputs
larger than the 126 MB L2 so no flush is needed between steps):
  reduce     fp32 row softmax + layernorm over 65536 x 4096 (x = 8 N(0,1),
             gamma N(1,0.1), beta N(0,0.1), eps 1e-5); a step is one softmax
             pass and one layernorm pass (independent: on two CUDA streams);
             metric GB/s moved (default, headline)
  gemm_u8s8  u8 x s8 GEMM M=16384 N=K=8192, zpA 128, per-channel requant to
             u8; metric TOPS (2 M N K per step)
  gemm_f16   fp16 GEMM M=N=K=8192, B column-major, fp32 accumulate; TFLOP/s
  attn       causal fp16 SDPA B=8 H=32 S=4096 D=128; TFLOP/s with the causal
             FLOP count 4 B H D S (S+1) / 2
  gemm_i8    int8 GEMM M=N=K=256 + requant (the CPU-runnable configuration)

With N > 1 (torchrun) the rows (M rows, or B*H heads) are split across the
ranks (strong scaling, no data-path collective); each rank times on its own
device with CUDA events and the job time is the max over ranks.
`--shard-of N` on one GPU times rank 0's part of an N-way split instead (the
per-rank problem of an N-GPU run, without the other ranks).

Rank 0 prints one JSON line.  `--impl reference` times the reference's scalar
CPU code (or its restatement where the reference has no such shape) on all
host cores for the same workload and prints the same line with
"impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

BASELINE_METRIC = "int8 GEMM TOPS, fp16 attn TFLOP/s, reduce GB/s; % roofline @1/2/4/8 B200"


# ------------------------------------------------------------------ helpers

def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    p = REPO / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class ClockSampler:
    """Polls NVML (SM clock, clock-event reasons) every 2 ms in a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, ordinal: int):
        self.ok = False
        self.samples = []
        self.reasons = 0
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(ordinal)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report nothing rather than guess
            self.err = str(e)

    def _run(self):
        nv = self.nvml
        while not self.stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.stop = threading.Event()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        med = float(np.median(self.samples)) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


class Dist:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        if gpus > 1 and self.world == 1:
            raise SystemExit(f"--gpus {gpus} needs torchrun with {gpus} processes")

    def init(self, backend: str):
        self.backend = backend
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            kw = {}
            if backend == "nccl":
                kw["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        import torch.distributed as dist
        dev = "cuda" if self.backend == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


def shard(total: int, world: int, rank: int):
    return total * rank // world, total * (rank + 1) // world


# ---------------------------------------------------------------- workloads

class Workload:
    """One benchmark configuration.  Subclasses define the per-rank device
    buffers, one step (device path), the host-API step (e2e) and a bounded CPU
    sample."""
    name = ""
    unit = ""
    dtype = ""
    bound = "hbm"

    def __init__(self, world=1, rank=0):
        self.world, self.rank = world, rank

    # total algorithmic units (bytes or ops) of one whole-job step
    def units_per_step(self) -> float:
        raise NotImplementedError

    def scale(self) -> float:
        return 1e9 if self.unit == "GB/s" else 1e12

    def gather_spec(self):
        """Outputs a replicated run all-gathers: (this rank's rows, total
        rows, bytes per row) each; None when the output does not shard."""
        return None


class Reduce(Workload):
    name = "reduce"
    unit = "GB/s"
    dtype = "f32"
    R, C, EPS = 65536, 4096, 1e-5
    # the step's softmax and layernorm are independent (both read x, each
    # writes its own output): they run on two CUDA streams, so one kernel's
    # launch gap and last-wave tail overlap the other's streaming
    streams = 2

    def config(self):
        return {"workload": "fp32 row softmax + layernorm 65536x4096", "rows": self.R,
                "cols": self.C, "eps": self.EPS, "x": "8*N(0,1)", "gamma": "N(1,0.1)",
                "beta": "N(0,0.1)", "seed": 0, "l2": "inputs 1 GiB > L2, no flush",
                "sharding": "rows", "parallelism": f"rows/{self.world}",
                "streams": "softmax and layernorm of a step on two CUDA streams"}

    def units_per_step(self):
        # softmax and layernorm each read R*C and write R*C fp32 (+ gamma, beta)
        return 2 * 2 * self.R * self.C * 4 + 2 * self.C * 4

    def host_inputs(self):
        r0, r1 = shard(self.R, self.world, self.rank)
        rng = np.random.default_rng(0)
        # generate only this rank's rows, deterministically per row block
        x = np.empty((r1 - r0, self.C), np.float32)
        blk = 4096
        for b0 in range(r0 - r0 % blk, r1, blk):
            xb = (np.random.default_rng([0, b0]).standard_normal((blk, self.C), dtype=np.float32) * 8)
            lo, hi = max(b0, r0), min(b0 + blk, r1)
            x[lo - r0:hi - r0] = xb[lo - b0:hi - b0]
        g = rng.normal(1, 0.1, self.C).astype(np.float32)
        b = rng.normal(0, 0.1, self.C).astype(np.float32)
        return x, g, b

    def setup_device(self, torch):
        x, g, b = self.host_inputs()
        self.nrows = x.shape[0]
        self.x = torch.from_numpy(x).cuda()
        self.g = torch.from_numpy(g).cuda()
        self.b = torch.from_numpy(b).cuda()
        self.o1 = torch.empty_like(self.x)
        self.o2 = torch.empty_like(self.x)
        self.hx_host = (x, g, b)

    def gather_spec(self):
        # (this rank's output rows, total rows, bytes per row) per output
        return [(self.o1, self.R, self.C * 4), (self.o2, self.R, self.C * 4)]

    def kernels(self):
        # (label, algorithmic units of one launch on this rank)
        per = 2 * self.nrows * self.C * 4
        return [("softmax_f32", per), ("layernorm_f32", per + 2 * self.C * 4)]

    def launch(self, device, k):
        if k == 0:
            device.launch("softmax_f32", 0, self.x, self.o1, self.nrows, self.C)
        else:
            device.launch("layernorm_f32", 0, self.x, self.g, self.b, self.o2, self.nrows, self.C,
                          self.EPS)

    # e2e through the public host API with pinned host buffers
    def setup_e2e(self, torch):
        x, g, b = self.hx_host
        self.px = torch.from_numpy(x).pin_memory()
        self.pg_ = torch.from_numpy(g).pin_memory()
        self.pb = torch.from_numpy(b).pin_memory()
        self.po1 = torch.empty_like(self.px).pin_memory()
        self.po2 = torch.empty_like(self.px).pin_memory()

    def e2e_step(self, lib, check):
        n = self.nrows
        check(lib.hexcuda_host_softmax_f32(self.px.data_ptr(), self.po1.data_ptr(), n, self.C))
        check(lib.hexcuda_host_layernorm_f32(self.px.data_ptr(), self.pg_.data_ptr(),
                                             self.pb.data_ptr(), self.po2.data_ptr(), n, self.C,
                                             self.EPS))

    def e2e_bytes(self):
        n = self.nrows
        return {"h2d_bytes_per_step": 2 * n * self.C * 4 + 2 * self.C * 4,
                "d2h_bytes_per_step": 2 * n * self.C * 4}

    def cpu_step(self, o, rows, nthreads):
        """Reference CPU code on `rows` rows; returns algorithmic bytes."""
        x = self.cpu_x[:rows]
        out = self.cpu_out[:rows]
        o.parallel(o.OP_SOFTMAX_F32, o.rows_args(x=x, out=out, R=rows, C=self.C), 0, rows, nthreads)
        o.parallel(o.OP_LAYERNORM_F32, o.rows_args(x=x, gamma=self.cpu_g, beta=self.cpu_b, out=out,
                                                   R=rows, C=self.C, eps=self.EPS), 0, rows,
                   nthreads)
        return 2 * 2 * rows * self.C * 4 + 2 * self.C * 4

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        self.cpu_x = (rng.standard_normal((rows, self.C), dtype=np.float32) * 8)
        self.cpu_out = np.empty_like(self.cpu_x)
        self.cpu_g = rng.normal(1, 0.1, self.C).astype(np.float32)
        self.cpu_b = rng.normal(0, 0.1, self.C).astype(np.float32)

    cpu_kind = "port"
    cpu_what = ("oracle/hexoracle.c restatement of fp16_softmax/reference.c:8-29 and "
                "fp16_layernorm/reference.c:7-24 in fp32 (the reference caps C at 256 / one row)")


class GemmU8S8(Workload):
    name = "gemm_u8s8"
    unit = "TOPS"
    dtype = "u8*s8->s32"
    bound = "tensor"
    M, N, K = 16384, 8192, 8192

    def config(self):
        return {"workload": "u8 x s8 GEMM 16384x8192x8192 per-channel requant to u8",
                "M": self.M, "N": self.N, "K": self.K, "zpA": 128, "zp_out": 128,
                "bias": "N(0,1000)", "mult": "[2^30,2^31)", "shift": 44, "seed": 0,
                "l2": "inputs 192 MiB > L2, no flush", "sharding": "M rows",
                "parallelism": f"M/{self.world}"}

    def units_per_step(self):
        return 2.0 * self.M * self.N * self.K

    def setup_device(self, torch):
        r0, r1 = shard(self.M, self.world, self.rank)
        self.m = r1 - r0
        g = torch.Generator(device="cuda").manual_seed(0)
        self.A = torch.randint(0, 256, (self.m, self.K), dtype=torch.uint8, device="cuda",
                               generator=g)
        self.B = torch.randint(-128, 128, (self.K, self.N), dtype=torch.int8, device="cuda",
                               generator=g)
        self.bias = torch.round(torch.randn(self.N, device="cuda", generator=g) * 1000).int()
        self.mult = torch.randint(2**30, 2**31 - 1, (self.N,), device="cuda", generator=g).int()
        self.shift = torch.full((self.N,), 44, dtype=torch.int32, device="cuda")
        self.out = torch.empty((self.m, self.N), dtype=torch.uint8, device="cuda")

    def gather_spec(self):
        return [(self.out, self.M, self.N)]

    def kernels(self):
        return [("gemm_u8s8_pc", 2.0 * self.m * self.N * self.K)]

    def launch(self, device, k):
        device.launch("gemm_u8s8_pc", 0, self.A, self.B, self.bias, self.out, self.m, self.N,
                      self.K, 128, self.mult, self.shift, 128)

    def setup_e2e(self, torch):
        self.h = [t.cpu().pin_memory() for t in (self.A, self.B, self.bias, self.mult, self.shift)]
        self.hout = torch.empty((self.m, self.N), dtype=torch.uint8).pin_memory()

    def e2e_step(self, lib, check):
        A, B, bias, mult, shift = (t.data_ptr() for t in self.h)
        check(lib.hexcuda_host_gemm_u8s8_pc(A, B, bias, self.hout.data_ptr(), self.m, self.N,
                                            self.K, 128, mult, shift, 128))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": self.m * self.K + self.K * self.N + 3 * 4 * self.N,
                "d2h_bytes_per_step": self.m * self.N}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        self.cA = rng.integers(0, 256, (rows, self.K), dtype=np.uint8)
        self.cB = rng.integers(-128, 128, (self.K, self.N), dtype=np.int8)
        self.cbias = np.round(rng.normal(0, 1000, self.N)).astype(np.int32)
        self.cmult = rng.integers(2**30, 2**31, self.N, dtype=np.int64).astype(np.int32)
        self.cshift = np.full(self.N, 44, np.int32)
        self.cout = np.empty((rows, self.N), np.uint8)

    def cpu_step(self, o, rows, nthreads):
        a = o.gemm_args(A=self.cA, B=self.cB, bias=self.cbias, out=self.cout, M=rows, N=self.N,
                        K=self.K, zpA=128, zp=128, mult_pc=self.cmult, shift_pc=self.cshift)
        o.parallel(o.OP_GEMM_U8S8_PC, a, 0, rows, nthreads)
        return 2.0 * rows * self.N * self.K

    cpu_kind = "port"
    cpu_what = ("oracle restatement composing gemm_tile_zp_i8/reference.c:10-28, "
                "i8_gemm_bias_requant/reference.c:13, requant_per_channel/reference.c:4-15, "
                "requantize_i32_u8_dma/reference.c:5-13")


class GemmF16(Workload):
    name = "gemm_f16"
    unit = "TFLOP/s"
    dtype = "f16*f16->f32"
    bound = "tensor"
    M = N = K = 8192

    def config(self):
        return {"workload": "fp16 GEMM 8192^3 A row-major B column-major", "M": self.M,
                "N": self.N, "K": self.K, "entries": "N(0,1)/sqrt(K)", "seed": 0,
                "l2": "inputs 256 MiB > L2, no flush", "sharding": "M rows",
                "parallelism": f"M/{self.world}"}

    def units_per_step(self):
        return 2.0 * self.M * self.N * self.K

    def setup_device(self, torch):
        r0, r1 = shard(self.M, self.world, self.rank)
        self.m = r1 - r0
        g = torch.Generator(device="cuda").manual_seed(0)
        s = 1.0 / math.sqrt(self.K)
        self.A = (torch.randn((self.m, self.K), device="cuda", generator=g) * s).half()
        self.Bt = (torch.randn((self.N, self.K), device="cuda", generator=g) * s).half()
        self.out = torch.empty((self.m, self.N), dtype=torch.float16, device="cuda")

    def gather_spec(self):
        return [(self.out, self.M, 2 * self.N)]

    def kernels(self):
        return [("gemm_f16_nt", 2.0 * self.m * self.N * self.K)]

    def launch(self, device, k):
        device.launch("gemm_f16_nt", 0, self.A, self.Bt, self.out, self.m, self.N, self.K)

    def setup_e2e(self, torch):
        self.h = [t.cpu().pin_memory() for t in (self.A, self.Bt)]
        self.hout = torch.empty((self.m, self.N), dtype=torch.float16).pin_memory()

    def e2e_step(self, lib, check):
        check(lib.hexcuda_host_gemm_f16_nt(self.h[0].data_ptr(), self.h[1].data_ptr(),
                                           self.hout.data_ptr(), self.m, self.N, self.K))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": 2 * (self.m * self.K + self.N * self.K),
                "d2h_bytes_per_step": 2 * self.m * self.N}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        s = 1.0 / math.sqrt(self.K)
        self.cA = (rng.standard_normal((rows, self.K), dtype=np.float32) * s).astype(np.float16)
        self.cB = (rng.standard_normal((self.N, self.K), dtype=np.float32) * s).astype(np.float16)
        self.cout = np.empty((rows, self.N), np.float16)

    def cpu_step(self, o, rows, nthreads):
        a = o.gemm_args(A=self.cA, B=self.cB, out=self.cout, M=rows, N=self.N, K=self.K)
        o.parallel(o.OP_GEMM_F16_NT, a, 0, rows, nthreads)
        return 2.0 * rows * self.N * self.K

    cpu_kind = "port"
    cpu_what = "oracle restatement of fp16_attention_qkt_hmx/reference.c:8-14 (M x N x K)"


class Attn(Workload):
    name = "attn"
    unit = "TFLOP/s"
    dtype = "f16, f32 softmax"
    bound = "tensor"
    B, H, S, D = 8, 32, 4096, 128

    def config(self):
        return {"workload": "causal fp16 SDPA B=8 H=32 S=4096 D=128", "B": self.B, "H": self.H,
                "S": self.S, "D": self.D, "scale": 1 / math.sqrt(self.D), "causal": True,
                "qkv": "N(0,1)", "seed": 0, "l2": "inputs 768 MiB > L2, no flush",
                "sharding": "B*H heads", "parallelism": f"heads/{self.world}",
                "flop_count": "causal: 4*B*H*D*S*(S+1)/2"}

    def flops(self, heads):
        return 4.0 * heads * self.D * self.S * (self.S + 1) / 2

    def units_per_step(self):
        return self.flops(self.B * self.H)

    def setup_device(self, torch):
        h0, h1 = shard(self.B * self.H, self.world, self.rank)
        self.h = h1 - h0
        g = torch.Generator(device="cuda").manual_seed(0)
        shp = (self.h, self.S, self.D)
        self.Q = torch.randn(shp, device="cuda", generator=g).half()
        self.K_ = torch.randn(shp, device="cuda", generator=g).half()
        self.V = torch.randn(shp, device="cuda", generator=g).half()
        self.O = torch.empty_like(self.Q)

    def gather_spec(self):
        return [(self.O, self.B * self.H, 2 * self.S * self.D)]

    def kernels(self):
        return [("attn_f16", self.flops(self.h))]

    def launch(self, device, k):
        device.launch("attn_f16", 0, self.Q, self.K_, self.V, self.O, self.h, self.S, self.S,
                      self.D, 1 / math.sqrt(self.D), 1)

    def setup_e2e(self, torch):
        self.hq = [t.cpu().pin_memory() for t in (self.Q, self.K_, self.V)]
        self.hout = torch.empty_like(self.hq[0]).pin_memory()

    def e2e_step(self, lib, check):
        q, k, v = (t.data_ptr() for t in self.hq)
        check(lib.hexcuda_host_attn_f16(q, k, v, self.hout.data_ptr(), self.h, self.S, self.S,
                                        self.D, 1 / math.sqrt(self.D), 1))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": 3 * 2 * self.h * self.S * self.D,
                "d2h_bytes_per_step": 2 * self.h * self.S * self.D}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        shp = (1, self.S, self.D)
        self.cQ, self.cK, self.cV = (rng.standard_normal(shp, dtype=np.float32).astype(np.float16)
                                     for _ in range(3))
        self.cO = np.empty_like(self.cQ)

    def cpu_step(self, o, rows, nthreads):
        # `rows` query rows of one head, spread over the causal triangle
        a = o.attn_args(Q=self.cQ, K=self.cK, V=self.cV, O=self.cO, BH=1, SQ=self.S, SK=self.S,
                        D=self.D, scale=1 / math.sqrt(self.D), causal=1)
        q0 = self.S - rows
        o.parallel(o.OP_ATTN_F16, a, q0, self.S, nthreads)
        keys = sum(i + 1 for i in range(q0, self.S))
        return 4.0 * self.D * keys

    cpu_kind = "port"
    cpu_what = ("oracle restatement of fp16_flash_attention_tile/reference.c:9-28 with causal "
                "window and scale parameter")


class GemmI8(Workload):
    name = "gemm_i8"
    unit = "TOPS"
    dtype = "s8*s8->s32"
    bound = "tensor"
    M = N = K = 256

    def config(self):
        return {"workload": "int8 GEMM 256^3 + requant (mult [2^30,2^31), shift 8..15)",
                "M": 256, "N": 256, "K": 256, "seed": 0, "l2": "fits in L2 (launch-bound)",
                "sharding": "none (replicas)", "parallelism": f"replicas/{self.world}"}

    def units_per_step(self):
        return 2.0 * self.M * self.N * self.K * self.world

    def setup_device(self, torch):
        rng = np.random.default_rng(0)
        A = rng.integers(-128, 128, (256, 256), dtype=np.int8)
        B = rng.integers(-128, 128, (256, 256), dtype=np.int8)
        self.mult = int(rng.integers(2**30, 2**31))
        self.shift = int(rng.integers(8, 16))
        self.A, self.B = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        self.out = torch.empty((256, 256), dtype=torch.int8, device="cuda")

    def kernels(self):
        return [("gemm_i8_requant", 2.0 * 256 ** 3)]

    def launch(self, device, k):
        device.launch("gemm_i8_requant", 0, self.A, self.B, self.out, 256, 256, 256, self.mult,
                      self.shift, 0)

    def setup_e2e(self, torch):
        self.h = [t.cpu().pin_memory() for t in (self.A, self.B)]
        self.hout = torch.empty((256, 256), dtype=torch.int8).pin_memory()

    def e2e_step(self, lib, check):
        check(lib.hexcuda_host_gemm_i8_requant(self.h[0].data_ptr(), self.h[1].data_ptr(),
                                               self.hout.data_ptr(), 256, 256, 256, self.mult,
                                               self.shift, 0))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": 2 * 256 * 256, "d2h_bytes_per_step": 256 * 256}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        self.cA = rng.integers(-128, 128, (256, 256), dtype=np.int8)
        self.cB = rng.integers(-128, 128, (256, 256), dtype=np.int8)
        self.cout = np.empty((256, 256), np.int8)

    def cpu_step(self, o, rows, nthreads):
        ref = o.ref_lib()
        if ref is not None:
            import ctypes as C
            ref.ref_i8_gemm_requant(self.cA.ctypes.data, self.cB.ctypes.data, self.cout.ctypes.data,
                                    256, 256, 256, C.c_int32(1 << 30), C.c_int(10), C.c_int8(0))
        else:
            a = o.gemm_args(A=self.cA, B=self.cB, out=self.cout, M=256, N=256, K=256,
                            mult=1 << 30, shift=10, zp=0)
            o.parallel(o.OP_I8_GEMM_REQUANT, a, 0, 256, 1)
        return 2.0 * 256 ** 3

    @property
    def cpu_kind(self):
        from oracle import oracle as o
        return "reference" if o.ref_lib() is not None else "port"

    cpu_what = "kernels/expert/i8_gemm_requant/reference.c (one thread)"


def _threaded(fn, total, nthreads):
    """Run fn(r0, r1) over [0, total) split across nthreads host threads (the
    oracle's C calls release the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    parts = [(total * i // nthreads, total * (i + 1) // nthreads) for i in range(nthreads)]
    with ThreadPoolExecutor(nthreads) as ex:
        list(ex.map(lambda p: fn(*p), [p for p in parts if p[1] > p[0]]))


class RequantEw(Workload):
    """residual_add_requant over 2^28 int32 pairs (the elementwise requant
    kernel's two-input form): HBM-bound, 9 bytes per element."""
    name = "requant"
    unit = "GB/s"
    dtype = "int64"
    bound = "hbm"
    N = 1 << 28
    MULT, SHIFT, ZP = 1518500250, 38, 3

    def config(self):
        return {"workload": "residual_add_requant int32+int32 -> int8, 2^28 elements",
                "n": self.N, "a": "U[-2^30,2^30)", "b": "U[-2^30,2^30)", "mult": self.MULT,
                "shift": self.SHIFT, "zp": self.ZP, "seed": 0,
                "l2": "inputs 2 GiB > L2, no flush", "sharding": "elements",
                "parallelism": f"elements/{self.world}"}

    def units_per_step(self):
        return 9.0 * self.N

    def setup_device(self, torch):
        r0, r1 = shard(self.N, self.world, self.rank)
        self.n = r1 - r0
        g = torch.Generator(device="cuda").manual_seed(0)
        self.a = torch.randint(-2**30, 2**30, (self.n,), dtype=torch.int32, device="cuda", generator=g)
        self.b = torch.randint(-2**30, 2**30, (self.n,), dtype=torch.int32, device="cuda", generator=g)
        self.out = torch.empty((self.n,), dtype=torch.int8, device="cuda")

    def gather_spec(self):
        return [(self.out, self.N, 1)]

    def kernels(self):
        return [("requant_ew", 9.0 * self.n)]

    def launch(self, device, k):
        device.launch("requant_ew", 0, self.a, 0, self.b, 1, self.out, self.n, 1, 0, self.MULT,
                      self.SHIFT, self.ZP, 0, -128, 127, -128, 127, None)

    def setup_e2e(self, torch):
        self.h = [t.cpu().pin_memory() for t in (self.a, self.b)]
        self.hout = torch.empty((self.n,), dtype=torch.int8).pin_memory()

    def e2e_step(self, lib, check):
        check(lib.hexcuda_host_requant_ew(self.h[0].data_ptr(), 0, self.h[1].data_ptr(), 1,
                                          self.hout.data_ptr(), self.n, 1, 0, self.MULT,
                                          self.SHIFT, self.ZP, 0, -128, 127, -128, 127, None))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": 8 * self.n, "d2h_bytes_per_step": self.n}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        self.ca = rng.integers(-2**30, 2**30, rows).astype(np.int32)
        self.cb = rng.integers(-2**30, 2**30, rows).astype(np.int32)
        self.cout = np.empty(rows, np.int8)

    def cpu_step(self, o, rows, nthreads):
        import ctypes as C
        ref = o.ref_lib()
        lib = o.lib()

        def part(r0, r1):
            a = C.c_void_p(self.ca.ctypes.data + 4 * r0)
            b = C.c_void_p(self.cb.ctypes.data + 4 * r0)
            out = C.c_void_p(self.cout.ctypes.data + r0)
            if ref is not None:
                # the reference's own reference.c, each thread on its slice
                ref.ref_residual_add_requant(a, b, out, C.c_int(r1 - r0), C.c_int32(self.MULT),
                                             C.c_int(self.SHIFT), C.c_int8(self.ZP))
            else:
                lib.oracle_requant_ew(a, 0, b, 1, C.c_int64(r1 - r0), 1, C.c_int64(0),
                                      C.c_int32(self.MULT), self.SHIFT, self.ZP, 0, -128, 127,
                                      -128, 127, None, out)
        _threaded(part, rows, nthreads)
        return 9.0 * rows

    @property
    def cpu_kind(self):
        from oracle import oracle as o
        return "reference" if o.ref_lib() is not None else "port"

    cpu_what = ("kernels/expert/residual_add_requant/reference.c (or its oracle/hexoracle.c "
                "restatement where the reference is not built), one slice per thread")


class ReduceI8(Workload):
    """i8_sum_dma at scale: the int32 sum of 2^31 int8 (2 GiB read once) on
    the integer whole-array reduction kernel; HBM-bound, 1 byte per element."""
    name = "reduce_i8"
    unit = "GB/s"
    dtype = "int32"
    bound = "hbm"
    N = 1 << 31

    def config(self):
        return {"workload": "i8_sum_dma: int32 sum of 2^31 int8", "n": self.N,
                "a": "U[-128,128)", "seed": 0, "l2": "input 2 GiB > L2, no flush",
                "sharding": "elements", "parallelism": f"elements/{self.world}"}

    def units_per_step(self):
        return float(self.N)

    def setup_device(self, torch):
        r0, r1 = shard(self.N, self.world, self.rank)
        self.n = r1 - r0
        g = torch.Generator(device="cuda").manual_seed(0)
        self.a = torch.randint(-128, 128, (self.n,), dtype=torch.int8, device="cuda", generator=g)
        self.out = torch.zeros(2, dtype=torch.int32, device="cuda")

    def kernels(self):
        return [("reduce_int", float(self.n))]

    def launch(self, device, k):
        device.launch("reduce_int", 0, self.a, None, 0, self.n, 0, self.out)

    def setup_e2e(self, torch):
        self.h = self.a.cpu().pin_memory()
        self.hout = torch.zeros(2, dtype=torch.int32).pin_memory()

    def e2e_step(self, lib, check):
        check(lib.hexcuda_host_reduce_int(self.h.data_ptr(), None, 0, self.n, 0,
                                          self.hout.data_ptr()))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": self.n, "d2h_bytes_per_step": 4}

    def cpu_setup(self, rows):
        self.ca = np.random.default_rng(0).integers(-128, 128, rows, dtype=np.int8)
        self.cout = np.zeros(256, np.int32)

    def cpu_step(self, o, rows, nthreads):
        import ctypes as C
        ref = o.ref_lib()
        lib = o.lib()

        def part(r0, r1):
            slot = min(255, r0 * max(1, nthreads) // max(1, rows))
            a = C.c_void_p(self.ca.ctypes.data + r0)
            out = C.c_void_p(self.cout.ctypes.data + 4 * slot)
            if ref is not None:
                # the reference's own reference.c, each thread on its slice
                ref.ref_i8_sum_dma(a, C.c_int(r1 - r0), out)
            else:
                lib.oracle_reduce_int(a, None, 0, C.c_int64(r1 - r0), 0, out)
        _threaded(part, rows, nthreads)
        return float(rows)

    @property
    def cpu_kind(self):
        from oracle import oracle as o
        return "reference" if o.ref_lib() is not None else "port"

    cpu_what = ("kernels/expert/i8_sum_dma/reference.c (or its oracle/hexoracle.c restatement "
                "where the reference is not built), one slice per thread, int32 partial sums")


class GemmHmx(Workload):
    """HMX-convention u8 x s8 GEMM with bias and ReLU to int32
    (i8_matmul_bias_relu_hmx's epilogue) at 16384 x 8192 x 8192."""
    name = "gemm_hmx"
    unit = "TOPS"
    dtype = "u8*s8->s32"
    bound = "tensor"
    M, N, K = 16384, 8192, 8192

    def config(self):
        return {"workload": "HMX-convention u8 x s8 GEMM 16384x8192x8192, sx12 + bias + ReLU -> int32",
                "M": self.M, "N": self.N, "K": self.K, "bias": "U[-3000,3000)", "seed": 0,
                "l2": "inputs 192 MiB > L2, no flush", "sharding": "M rows",
                "parallelism": f"M/{self.world}"}

    def units_per_step(self):
        return 2.0 * self.M * self.N * self.K

    def setup_device(self, torch):
        r0, r1 = shard(self.M, self.world, self.rank)
        self.m = r1 - r0
        g = torch.Generator(device="cuda").manual_seed(0)
        self.A = torch.randint(0, 256, (self.m, self.K), dtype=torch.uint8, device="cuda", generator=g)
        self.B = torch.randint(-128, 128, (self.K, self.N), dtype=torch.int8, device="cuda", generator=g)
        self.bias = torch.randint(-3000, 3000, (self.N,), dtype=torch.int32, device="cuda", generator=g)
        self.out = torch.empty((self.m, self.N), dtype=torch.int32, device="cuda")

    def gather_spec(self):
        return [(self.out, self.M, 4 * self.N)]

    def kernels(self):
        return [("gemm_hmx_ex", 2.0 * self.m * self.N * self.K)]

    def launch(self, device, k):
        device.launch("gemm_hmx_ex", 0, self.A, self.B, 0, self.bias, None, 0, None, self.out, 0, 1,
                      0, self.m, self.N, self.K, 0)

    def setup_e2e(self, torch):
        self.h = [t.cpu().pin_memory() for t in (self.A, self.B, self.bias)]
        self.hout = torch.empty((self.m, self.N), dtype=torch.int32).pin_memory()

    def e2e_step(self, lib, check):
        A, B, bias = (t.data_ptr() for t in self.h)
        check(lib.hexcuda_host_gemm_hmx_ex(A, B, 0, bias, None, 0, None, self.hout.data_ptr(), 0,
                                           1, 0, self.m, self.N, self.K, 0))

    def e2e_bytes(self):
        return {"h2d_bytes_per_step": self.m * self.K + self.K * self.N + 4 * self.N,
                "d2h_bytes_per_step": 4 * self.m * self.N}

    def cpu_setup(self, rows):
        rng = np.random.default_rng(0)
        self.cA = rng.integers(0, 256, (rows, self.K), dtype=np.uint8)
        self.cB = rng.integers(-128, 128, (self.K, self.N), dtype=np.int8)
        self.cbias = rng.integers(-3000, 3000, self.N).astype(np.int32)
        self.cout = np.empty((rows, self.N), np.int32)

    def cpu_step(self, o, rows, nthreads):
        import ctypes as C
        lib = o.lib()

        def part(r0, r1):
            lib.oracle_gemm_hmx_ex_rows(C.c_void_p(self.cA.ctypes.data), C.c_void_p(self.cB.ctypes.data),
                                        0, C.c_void_p(self.cout.ctypes.data), rows, self.N, self.K,
                                        C.c_int32(0), 0, 1, C.c_void_p(self.cbias.ctypes.data), 0,
                                        None, None, 0, r0, r1)
        _threaded(part, rows, nthreads)
        return 2.0 * rows * self.N * self.K

    cpu_kind = "port"
    cpu_what = ("oracle/hexoracle.c restatement of the HMX-convention GEMMs "
                "(i8_matmul_bias_relu_hmx/reference.c), rows split over host threads")


# short workload names of the extra ops in the bench line (full configs:
# `python bench.py --workload NAME --ops none`)
OP_LABELS = {"gemm_u8s8": "u8s8 GEMM 16384x8192x8192 pc-requant", "gemm_f16": "f16 GEMM 8192^3 NT",
             "attn": "causal SDPA 8x32x4096x128", "gemm_i8": "i8 GEMM 256^3 requant",
             "requant": "residual_add_requant 2^28", "gemm_hmx": "HMX GEMM 16384x8192x8192 i32",
             "reduce_i8": "i8_sum 2^31"}

WORKLOADS = {w.name: w for w in (Reduce, GemmU8S8, GemmF16, Attn, GemmI8, RequantEw, GemmHmx,
                                  ReduceI8)}


# ------------------------------------------------------------------- timing

def time_device(wl, torch, device, steps, warmup, dist, lib):
    """Timed region: barrier + sync, K steps back to back on torch's current
    stream between one start and one end CUDA event, sync + barrier.  An
    event recorded between launches costs a few microseconds of stream time,
    so the library's own per-launch events are off here; a second pass of the
    same K steps with an event pair around each launch splits the step time
    between the kernels (for the roofline).  Returns a dict."""
    kernels = wl.kernels()
    for _ in range(warmup):
        for k in range(len(kernels)):
            wl.launch(device, k)
    torch.cuda.synchronize()
    device.sync(0)
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream() if getattr(wl, "streams", 1) > 1 else None

    def launch_step():
        for k in range(len(kernels)):
            if side is not None and k % 2 == 1:
                device.bind_stream(0, side)
                wl.launch(device, k)
                device.bind_stream(0, stream)
            else:
                wl.launch(device, k)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lib.hexcuda_set_timing(0)
    try:
        launches0 = lib.hexcuda_launch_count()
        dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(torch.cuda.current_device()) as clk:
            start.record(stream)
            if side is not None:
                side.wait_event(start)
            for s in range(steps):
                launch_step()
            if side is not None:
                joined = torch.cuda.Event()
                joined.record(side)
                stream.wait_event(joined)
            end.record(stream)
            torch.cuda.synchronize()
        dist.barrier()
        device.sync(0)
        launches = lib.hexcuda_launch_count() - launches0
        ms = start.elapsed_time(end)
        # per-kernel durations: the same steps, one event pair per launch
        ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in kernels] for _ in range(steps)]
        for s in range(steps):
            for k in range(len(kernels)):
                ev[s][k][0].record(stream)
                wl.launch(device, k)
                ev[s][k][1].record(stream)
        torch.cuda.synchronize()
        device.sync(0)
    finally:
        lib.hexcuda_set_timing(1)
    # A kernel's duration: its share of the event-free step (the second pass
    # only splits the step between the kernels; it runs later, on a GPU that
    # may have settled to lower power-capped clocks, and with event overhead)
    raw = [float(np.mean([ev[s][k][0].elapsed_time(ev[s][k][1]) for s in range(steps)]))
           for k in range(len(kernels))]
    per_kernel = [(label, units, ms / steps * raw[k] / sum(raw))
                  for k, (label, units) in enumerate(kernels)]
    return {"ms": ms, "per_kernel": per_kernel, "clocks": clk.summary(), "launches": launches}


def time_e2e(wl, torch, lib, check, steps, warmup, dist):
    wl.setup_e2e(torch)
    for _ in range(max(1, warmup // 2)):
        wl.e2e_step(lib, check)
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        wl.e2e_step(lib, check)
    dt = time.perf_counter() - t0
    return dt


def cpu_measure(wl, budget_s: float, nthreads: int, max_rows: int):
    """Bounded CPU sample: grows the sample until one call takes ~budget/4,
    then times repeated calls for about `budget_s` seconds."""
    from oracle import oracle as o
    o.lib()
    rows = {"reduce": 256, "requant": 1 << 16, "reduce_i8": 1 << 22}.get(wl.name, 8)
    rows = min(rows, max_rows)
    while True:
        wl.cpu_setup(rows)
        t0 = time.perf_counter()
        units = wl.cpu_step(o, rows, nthreads)
        dt = time.perf_counter() - t0
        if dt > budget_s / 4 or rows >= max_rows:
            break
        rows = min(max_rows, rows * 4)
    reps, tot, units_tot = 0, 0.0, 0.0
    while tot < budget_s * 0.75 or reps < 1:
        t0 = time.perf_counter()
        units_tot += wl.cpu_step(o, rows, nthreads)
        tot += time.perf_counter() - t0
        reps += 1
    return units_tot / tot, rows, reps, tot


def cpu_rows_cap(wl):
    return {"reduce": wl.R if hasattr(wl, "R") else 0, "gemm_u8s8": 4096, "gemm_f16": 4096,
            "attn": 4096, "gemm_i8": 256, "requant": 1 << 28, "gemm_hmx": 4096,
            "reduce_i8": 1 << 28}[wl.name]


def cpu_sample_text(wl, rows, reps, secs):
    if wl.name == "reduce":
        return f"{rows} of 65536 rows, softmax+layernorm, {reps} reps, {secs:.1f} s"
    if wl.name == "attn":
        return f"last {rows} query rows of one causal head (S=4096, D=128), {reps} reps, {secs:.1f} s"
    if wl.name == "gemm_i8":
        return f"the full 256^3 GEMM, {reps} reps, {secs:.1f} s"
    if wl.name == "requant":
        return f"{rows} of 2^28 elements, {reps} reps, {secs:.1f} s"
    if wl.name == "reduce_i8":
        return f"{rows} of 2^31 elements, {reps} reps, {secs:.1f} s"
    return f"{rows} rows of M with full N, K, {reps} reps, {secs:.1f} s"


# --------------------------------------------------------------------- arms

def measure_pcie(torch, nbytes=256 << 20):
    """Pinned host <-> device copy bandwidth of this rank's GPU (GB/s): H2D
    alone, D2H alone, and both directions at once on two streams."""
    h_src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    h_dst = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_a = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    d_b = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s2 = torch.cuda.Stream()

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / reps

    def both():
        d_a.copy_(h_src, non_blocking=True)
        with torch.cuda.stream(s2):
            h_dst.copy_(d_b, non_blocking=True)

    h2d = nbytes / timed(lambda: d_a.copy_(h_src, non_blocking=True)) / 1e9
    d2h = nbytes / timed(lambda: h_dst.copy_(d_b, non_blocking=True)) / 1e9
    duplex = 2 * nbytes / timed(both) / 1e9
    return {"h2d_gbs": round(h2d, 1), "d2h_gbs": round(d2h, 1), "duplex_gbs": round(duplex, 1)}


def time_allgather(wl, torch, lib, check, steps, warmup, dist):
    """The replicated-output option: each output's row shards all-gathered
    across the ranks (NCCL over NVLink through hexcuda_comm_allgather_rows),
    timed on its own with CUDA events, max over ranks."""
    spec = wl.gather_spec()
    fulls = [torch.empty((rows, rb), dtype=torch.uint8, device="cuda") for _, rows, rb in spec]

    def step():
        for (shard, rows, rb), full in zip(spec, fulls):
            check(lib.hexcuda_comm_allgather_rows(shard.data_ptr(), full.data_ptr(), rows, rb))

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(start.elapsed_time(end)) / steps
    total = sum(rows * rb for _, rows, rb in spec)
    algbw = total / (ms / 1e3) / 1e9
    del fulls
    return {"ms_per_step": round(ms, 4), "bytes_per_step": total,
            "algbw_gbs": round(algbw, 1),
            "busbw_gbs": round(algbw * (dist.world - 1) / dist.world, 1),
            "api": "hexcuda_comm_allgather_rows (ncclAllGather, or one ncclBroadcast per "
                   "ragged part)"}


def run_ours(args, dist):
    import torch

    from hexkernels_b200 import _lib, device, ops

    torch.cuda.set_device(dist.local)
    lib = _lib.load()
    ops.init_devices([dist.local])
    # one dedicated stream carries both torch's work and libhexcuda's launches,
    # so the CUDA events recorded on it bracket exactly the timed kernels
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    device.bind_stream(0, stream)
    peaks = load_peaks()
    traffic = load_traffic()
    check = _lib.check
    replicate = args.replicate and dist.world > 1
    if replicate:
        import ctypes as C

        import torch.distributed as tdist
        uid = C.create_string_buffer(128)
        if dist.rank == 0:
            check(lib.hexcuda_comm_unique_id(uid, 128))
        box = [uid.raw if dist.rank == 0 else None]
        tdist.broadcast_object_list(box, src=0)
        C.memmove(uid, box[0], 128)
        check(lib.hexcuda_comm_init_rank(dist.world, dist.rank, uid, 128))

    # --shard-of N: this one GPU times rank 0's part of an N-way row split
    wl_world, wl_rank = ((args.shard_of, 0) if args.shard_of > 1 and dist.world == 1
                         else (dist.world, dist.rank))

    def measure(wl_cls, steps, cpu_budget):
        wl = wl_cls(wl_world, wl_rank)
        wl.setup_device(torch)
        t = time_device(wl, torch, device, steps, args.warmup, dist, lib)
        ms_max = dist.max(t["ms"])
        per_step_ms = ms_max / steps
        value = wl.units_per_step() / (per_step_ms / 1e3) / wl.scale()
        # dominant kernel roofline (this rank's launches)
        label, units, dur = max(t["per_kernel"], key=lambda r: r[2])
        achieved = units / (dur / 1e3) / wl.scale()
        if wl.bound == "hbm":
            peak, punit, pname = peaks["hbm_gbs"], "GB/s", "hbm_gbs"
        else:
            # int8 peaks are not measured by the driver: the dense int8 rate is
            # twice the dense bf16 rate on this part, so the int8 roofline is
            # 2x the measured bf16 figure
            mul = 2.0 if wl.unit == "TOPS" else 1.0
            peak, punit, pname = peaks["bf16_tflops"] * mul, wl.unit, "bf16_tflops"
        tr = traffic.get(label)
        res = {
            "metric": BASELINE_METRIC, "value": round(value, 3), "unit": wl.unit,
            "steps": steps, "ms_per_step": round(per_step_ms, 4), "dtype": wl.dtype,
            "config": wl.config(),
            "roofline": {"bound": wl.bound, "kernel": label, "achieved": round(achieved, 2),
                         "peak": peak, "unit": punit if wl.bound == "tensor" else "GB/s",
                         "frac": round(achieved / peak, 4),
                         "peak_source": f"{peaks['source']} {pname}" +
                                        (" x2 (int8 = 2x bf16 dense)" if wl.unit == "TOPS" else ""),
                         "traffic": (round(tr["bytes_per_launch"] * units / tr["units"])
                                     if tr else None),
                         "kernel_ms": round(dur, 4)},
            "clocks": t["clocks"], "gpu_launches": int(t["launches"]),
        }
        if hasattr(wl, "setup_e2e"):
            nst = max(2, min(steps, 20) // 4)
            dt = dist.max(time_e2e(wl, torch, lib, check, nst, args.warmup, dist))
            res["e2e"] = {"value": round(wl.units_per_step() / (dt / nst) / wl.scale(), 3),
                          "unit": wl.unit, **wl.e2e_bytes(), "steps": nst,
                          "api": "hexcuda_host_* (the candidate_kernel shims' call), pinned "
                                 "host buffers"}
        if replicate and wl.gather_spec() is not None:
            res["replicate"] = time_allgather(wl, torch, lib, check, max(3, steps // 2),
                                              args.warmup, dist)
        if cpu_budget > 0 and dist.rank == 0 and dist.world == 1:
            nthreads = len(os.sched_getaffinity(0))
            if wl.name == "gemm_i8":
                nthreads = 1
            v, rows, reps, secs = cpu_measure(wl, cpu_budget, nthreads, cpu_rows_cap(wl))
            res["cpu_baseline"] = {"value": round(v / wl.scale(), 6), "unit": wl.unit,
                                   "cores": nthreads, "kind": wl.cpu_kind,
                                   "sample": cpu_sample_text(wl, rows, reps, secs),
                                   "code": wl.cpu_what}
        del wl
        torch.cuda.empty_cache()
        return res

    pcie = measure_pcie(torch)
    head = measure(WORKLOADS[args.workload], args.steps, args.cpu_budget)
    if "e2e" in head:
        # the host-API number against what the copies alone allow on this link
        e = head["e2e"]
        gb_in, gb_out = e["h2d_bytes_per_step"] / 1e9, e["d2h_bytes_per_step"] / 1e9
        t_copy = max(gb_in / pcie["h2d_gbs"], gb_out / pcie["d2h_gbs"],
                     (gb_in + gb_out) / pcie["duplex_gbs"])
        wl0 = WORKLOADS[args.workload](wl_world, wl_rank)
        e["pcie"] = dict(pcie, ceiling=round(wl0.units_per_step() / t_copy / wl0.scale(), 3))
    ops_out = {}
    if args.ops == "all":
        for name in ("gemm_u8s8", "gemm_f16", "attn", "gemm_i8", "requant", "gemm_hmx",
                     "reduce_i8"):
            if name == args.workload:
                continue
            r = measure(WORKLOADS[name], max(args.steps, args.op_steps), args.op_cpu_budget)
            rf = r["roofline"]
            # compact, so that the whole line fits a log tail of ~3 KB
            entry = {"value": r["value"], "unit": r["unit"], "ms": r["ms_per_step"],
                     "steps": r["steps"], "workload": OP_LABELS[name],
                     "roofline": {k: rf[k] for k in ("kernel", "achieved", "peak", "frac")},
                     "sm_mhz": r["clocks"].get("sm_mhz"), "reasons": r["clocks"].get("reasons"),
                     "launches": r["gpu_launches"]}
            if "e2e" in r:
                entry["e2e"] = r["e2e"]["value"]
            if "cpu_baseline" in r:
                entry["cpu_baseline"] = {"value": r["cpu_baseline"]["value"],
                                         "kind": r["cpu_baseline"]["kind"]}
            if "replicate" in r:
                entry["allgather_busbw_gbs"] = r["replicate"]["busbw_gbs"]
            ops_out[name] = entry
    line = {"metric": head["metric"], "value": head["value"], "unit": head["unit"],
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "strong" if args.workload != "gemm_i8" else "weak",
            "vs_baseline": None, "dtype": head["dtype"], "data": "synthetic (seeded)",
            "config": head["config"], "roofline": head["roofline"], "clocks": head["clocks"],
            "gpu_launches": head["gpu_launches"]}
    for k in ("e2e", "cpu_baseline", "replicate"):
        if k in head:
            line[k] = head[k]
    if ops_out:
        line["ops"] = ops_out
    if wl_world != dist.world:
        line["shard_of"] = {"parts": wl_world, "timed": "rank 0's part on this GPU"}
    if replicate:
        check(lib.hexcuda_comm_destroy())
    return line


def run_reference(args, dist):
    """The reference's CPU implementation on this host's cores, same
    workload, bounded per-step samples."""
    wl = WORKLOADS[args.workload](1, 0)
    from oracle import oracle as o
    o.lib()
    nthreads = 1 if wl.name == "gemm_i8" else len(os.sched_getaffinity(0))
    # size the per-step sample so the whole run stays within ~2 minutes
    per_step_budget = max(0.2, 100.0 / max(1, args.steps + args.warmup))
    rows = {"reduce": 256, "requant": 1 << 16, "reduce_i8": 1 << 22}.get(wl.name, 8)
    cap = cpu_rows_cap(wl)
    while True:
        wl.cpu_setup(rows)
        t0 = time.perf_counter()
        wl.cpu_step(o, rows, nthreads)
        if time.perf_counter() - t0 > per_step_budget / 2 or rows >= cap:
            break
        rows = min(cap, rows * 2)
    for _ in range(args.warmup):
        wl.cpu_step(o, rows, nthreads)
    t0 = time.perf_counter()
    units = 0.0
    for _ in range(args.steps):
        units += wl.cpu_step(o, rows, nthreads)
    dt = time.perf_counter() - t0
    value = units / dt / wl.scale()
    sample = cpu_sample_text(wl, rows, args.steps, dt)
    return {"metric": BASELINE_METRIC, "value": round(value, 6), "unit": wl.unit, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded)", "config": wl.config(),
            "cpu_baseline": {"value": round(value, 6), "unit": wl.unit, "cores": nthreads,
                             "kind": wl.cpu_kind, "sample": sample, "code": wl.cpu_what},
            "e2e": {"value": round(value, 6), "unit": wl.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="reduce", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ops", default="all", choices=["all", "none"])
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work per cpu_baseline sample")
    ap.add_argument("--op-steps", type=int, default=50,
                    help="timed steps of each extra op (at least --steps)")
    ap.add_argument("--op-cpu-budget", type=float, default=2.5,
                    help="seconds of CPU work per extra op's cpu_baseline sample (0: none)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one GPU: time rank 0's row shard of an N-way split (the per-rank "
                         "problem of an N-GPU run); value = the whole problem's units over "
                         "that time")
    ap.add_argument("--replicate", action="store_true",
                    help="N > 1: also all-gather every sharded output over NCCL (timed apart)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    dist = Dist(args.gpus)
    if args.impl == "reference":
        if dist.rank == 0:
            print(json.dumps(run_reference(args, dist)), flush=True)
        return
    dist.init("nccl")
    try:
        line = run_ours(args, dist)
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
