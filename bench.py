"""Benchmark of phew's candidate-evaluation path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl phew|reference]
                    [--workload sweep|gelu_chain|attention|normed_matmul|
                                rms_norm|rms_norm_n256|rms_norm_n1024|qkv_proj|qk_scores|
                                softmax|score_softmax|score_softmax_8k|rms_rowmap]

Default workload (sweep): the verification sweep over a decoder block
(RMSNorm -> QKV projection (4096 = 32 heads x 128) -> causal attention ->
output projection -> SwiGLU MLP (hidden 14336), bf16, batch 8): the 16
candidate graphs the reference's passes emit for it, each verified against
the baseline over 5 seeds x 3 sizes (seq 512 / 2048 / 8192) x 4 edge
variants (zeros, N(0,1)*1e4, bf16 subnormals, one-hot rows) -- 960
candidate units and 60 baseline evaluations.  Processes (one per GPU) take
(seed, size, variant) groups from one host-side counter; there is no
data-path collective (strong scaling: the same sweep on 1..N GPUs).

Printed (one JSON line, rank 0):
  value       verified candidates / s: the 16 candidates over the device
              time of the whole sweep (max over ranks); the timed region is
              one full sweep, and a step is 1/K of it (ms_per_step = region / K)
  roofline    algorithmic FLOPs of the evaluated units (baselines and the
              candidates that ran to a comparison) per GPU-second, against
              the measured sustained bf16 GEMM peak
  e2e         the same sweep with every group's inputs drawn on the HOST
              (the counter-based generator on host threads, into pinned
              memory, one group ahead) and copied in, and every comparison
              record copied back
  cpu_baseline  the oracle (numpy restatement of the MLX-CPU evaluation) on a
              bounded sample of the 64-unit subset (16 candidates x seed 0 x
              seq 512 x 4 variants), extrapolated by FLOPs to the full sweep
  configs     (1 GPU) per-kernel figures of the other benchmark configs:
              rms_norm fp32 n = 256 / 1024 / 4096, the fused fp16 chain, causal
              SDPA bf16 (4,32,2048,128), normed matmul bf16 8192x4096x4096:
              value, roofline fraction, clocks and optimized_ms / baseline_ms

The other workloads print the same contract for one kernel: a step is one
launch over one batch of inputs resident in HBM (rotated past the 126 MB L2),
K launches captured in a CUDA graph and replayed inside the timed region;
e2e runs the public API with pinned host buffers (H2D and D2H every step).

``--impl reference`` times the reference's path on the host CPU (the oracle
port: MLX, the reference's runtime, is not installable here), using all
host threads, on the same workload and metric.  Under torchrun only rank 0
runs it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["phew", "reference"], default="phew")
    ap.add_argument("--workload", default="sweep", choices=["sweep", *WORKLOADS])
    # sweep options (the workload list includes sweep-internal kernels measured
    # on their own: qkv_proj, qk_scores, softmax, score_softmax, score_softmax_8k,
    # rms_rowmap)
    ap.add_argument("--seeds", type=int, default=5)
    ap.add_argument("--variants", choices=["edge", "reference"], default="edge")
    ap.add_argument("--tiny", action="store_true",
                    help="reduced decoder dimensions (a quick check, not a benchmark number)")
    ap.add_argument("--journal-dir", default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--cpu-units", type=int, default=32,
                    help="units of the CPU subset timed for cpu_baseline (32: two variants x "
                         "16 candidates, 10-20 s of CPU work on a 16-core host)")
    return ap.parse_args(argv)


def load_peaks() -> dict:
    """HBM copy GB/s and bf16 GEMM TFLOP/s (burst, and sustained for work
    timed inside a long step) measured on this pool's B200s, or the pool's
    earlier measurement when the file is absent."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic(name: str | None) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of this kernel
    and workload (profiles/<name>.traffic.json), or None."""
    if not name:
        return None
    p = ROOT / "profiles" / f"{name}.traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get("dram_bytes_per_launch")
    return None


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


class Dist:
    def __init__(self) -> None:
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.torch = torch
        self.dist = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        elif torch.cuda.is_available():
            torch.cuda.set_device(0)

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if not self.dist:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.dist:
            return v
        t = self.torch.tensor([float(v)], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.dist:
            self.dist.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index, self.proc, self.path = index, None, None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in Path(self.path).read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        except OSError:
            pass
        finally:
            if self.path:
                try:
                    os.unlink(self.path)
                except OSError:
                    pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------


def _opt_over_baseline(api, baseline_fn, opt_args, base_args) -> dict:
    """optimized_ms / baseline_ms: the substituted call (the optimizer's
    output) against the harness function evaluated op by op on this backend,
    both timed by phew_b200.bench (CUDA events, cold L2)."""
    from phew_b200.bench import benchmark

    opt = benchmark(lambda *a: api(list(a)), *opt_args, n_warmup=3, n_bench=10, max_n_bench=30)
    basel = benchmark(baseline_fn, *base_args, n_warmup=2, n_bench=5, max_n_bench=15)
    return {"optimized_ms": opt.mean_ms, "baseline_ms": basel.mean_ms,
            "optimized_over_baseline": opt.mean_ms / basel.mean_ms}


class GeluChain:
    """Fused elementwise chain, fp16 (4096, 8192): HBM-bound."""

    name = "gelu_chain"
    metric, unit, bound, dtype = "fused_kernel_hbm_gbs", "GB/s", "hbm", "f16"
    ROWS, COLS = 4096, 8192
    kernel_regex = "gelu_chain_fused"
    profile = "gelu_chain_fused_fp16_4096x8192"

    def describe(self):
        return (f"gelu_chain: z = tanh-GELU(x*a+b)*sigmoid(c)+x, fp16 ({self.ROWS},{self.COLS}), "
                "one fused NVRTC kernel per step")

    def work_per_step(self):
        from phew_b200.workloads import gelu_chain_bytes

        return gelu_chain_bytes(self.ROWS, self.COLS)

    def host_inputs(self, seed):
        from phew_b200.workloads import gelu_chain_inputs

        return gelu_chain_inputs("typical", seed)

    def setup(self, mx, host):
        import torch

        from phew_b200 import _native
        from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen
        from phew_b200.workloads import gelu_chain_nodes

        base = [mx.array(h) for h in host]
        self.sets = [base] + [[mx.array(a._t.clone()) for a in base] for _ in range(2)]
        chain, ins, outs = gelu_chain_nodes(self.ROWS, self.COLS)
        src, in_names, out_names = SubgraphCUDACodegen().emit(chain, ins, outs)
        self.kern = mx.fast.cuda_kernel("gelu_chain_fused", in_names, out_names, src)
        self.threads = mx.elementwise_threads(self.ROWS * self.COLS)
        self.outs = [mx.core.empty((self.ROWS, self.COLS), mx.float16) for _ in range(3)]
        self.api(self.sets[0])
        self.handle = next(iter(self.kern._handles.values()))
        self.argvs, self.keep = [], []
        for s, o in zip(self.sets, self.outs):
            vals = [ctypes.c_void_p(a._t.data_ptr()) for a in s + [o]]
            vals += [ctypes.c_uint64(a.size) for a in s + [o]]
            self.keep.append(vals)
            self.argvs.append((ctypes.c_void_p * len(vals))(
                *[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in vals]))
        self.lib = _native.load()
        self.blocks = -(-self.threads // 256)
        self.st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        self._native = _native

    def api(self, inputs):
        from phew_b200 import mx

        return self.kern(inputs=inputs, output_shapes=[(self.ROWS, self.COLS)],
                         output_dtypes=[mx.float16], grid=(self.threads, 1, 1),
                         threadgroup=(256, 1, 1))[0]

    def launch(self, i):
        import torch

        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = self.lib.phew_launch(ctypes.c_uint64(self.handle), self.argvs[i % 3], len(self.keep[0]),
                                  self.blocks, 1, 1, 256, 1, 1, 0, st)
        if rc:
            self._native.check(rc, "phew_launch")

    def extras(self, mx):
        from phew_b200.bench import benchmark
        from phew_b200.workloads import gelu_chain_fn

        opt = benchmark(lambda *a: self.api(list(a)), *self.sets[0], n_warmup=3, n_bench=10,
                        max_n_bench=30)
        basel = benchmark(gelu_chain_fn(mx), *self.sets[0], n_warmup=2, n_bench=5, max_n_bench=15)
        return {"optimized_ms": opt.mean_ms, "baseline_ms": basel.mean_ms,
                "optimized_over_baseline": opt.mean_ms / basel.mean_ms}

    def cpu_sample(self, threads: int, rows: int = 2048):
        from oracle import mlx_cpu
        from phew_b200.workloads import gelu_chain_bytes, gelu_chain_inputs, gelu_chain_nodes

        xs = gelu_chain_inputs("typical", 0, rows=rows)
        per = -(-rows // threads)
        parts = []
        for b in range(threads):
            lo, hi = b * per, min(rows, (b + 1) * per)
            if lo < hi:
                c, i, o = gelu_chain_nodes(hi - lo)
                parts.append((c, i, o, [xs[0][lo:hi], xs[1], xs[2], xs[3][lo:hi]]))
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(lambda p: mlx_cpu.eval_chain(*p), parts))
            t0 = time.perf_counter()
            list(ex.map(lambda p: mlx_cpu.eval_chain(*p), parts))
            dt = time.perf_counter() - t0
        return gelu_chain_bytes(rows) / dt / 1e9, dt, f"{rows} of {self.ROWS} rows"


class Attention:
    """Fused causal attention, bf16 (4, 32, 2048, 128): tensor-core bound."""

    name = "attention"
    metric, unit, bound, dtype = "sdpa_tflops", "TFLOP/s", "tensor", "bf16"
    B, H, L, D = 4, 32, 2048, 128
    kernel_regex = "sdpa_fwd"
    profile = "sdpa_fwd_causal_bf16_4x32x2048x128"
    scale = 1.0 / math.sqrt(128)

    def describe(self):
        return (f"causal SDPA softmax(q k^T / sqrt(128)) v, bf16 ({self.B},{self.H},{self.L},{self.D}), "
                "one tcgen05 kernel per step")

    def work_per_step(self):
        from phew_b200.workloads import attention_flops

        return attention_flops(self.B, self.H, self.L, self.D, causal=True)

    def host_inputs(self, seed):
        from phew_b200.workloads import attention_inputs

        return attention_inputs("typical", seed)[:3]

    def setup(self, mx, host):
        base = [mx.array(h) for h in host]
        self.sets = [base, [mx.array(a._t.clone()) for a in base]]
        self.api(self.sets[0])

    def api(self, inputs):
        from phew_b200 import mx

        return mx.fast.scaled_dot_product_attention(*inputs, scale=self.scale, mask="causal")

    def launch(self, i):
        self.api(self.sets[i % 2])

    def extras(self, mx):
        from phew_b200.workloads import attention_fn, causal_mask

        mask = mx.array(causal_mask(self.L))
        return _opt_over_baseline(self.api, attention_fn(mx), self.sets[0], self.sets[0] + [mask])

    def cpu_sample(self, threads: int):
        import numpy as np

        from oracle import mlx_cpu

        q, k, v = [h[:1, :threads] for h in self.host_inputs(0)]
        mlx_cpu.sdpa(*[mlx_cpu.array(x[:, :1]) for x in (q, k, v)], self.scale, "causal")
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(lambda h: mlx_cpu.sdpa(*[mlx_cpu.array(x[:, h:h + 1]) for x in (q, k, v)],
                                               self.scale, "causal"), range(q.shape[1])))
        dt = time.perf_counter() - t0
        flops = 2 * q.shape[1] * self.L * self.L * self.D
        _ = np
        return flops / dt / 1e12, dt, f"{q.shape[1]} of {self.B * self.H} heads"


class NormedMatmul:
    """(x @ W) * rsqrt(mean(x^2) + eps), bf16 8192 x 4096 x 4096: tensor-core bound."""

    name = "normed_matmul"
    metric, unit, bound, dtype = "normed_matmul_tflops", "TFLOP/s", "tensor", "bf16"
    M, K, N = 8192, 4096, 4096
    kernel_regex = "gemm_tc"
    profile = "gemm_tc_normed_matmul_bf16_8192x4096x4096"

    def describe(self):
        return (f"normed matmul (x @ W) * rsqrt(mean(x*x,-1)+1e-5), bf16 x ({self.M},{self.K}), "
                f"W ({self.K},{self.N}); a row-statistic pass over x, then one tcgen05 GEMM "
                f"applying the per-row factor in its epilogue (timed together)")

    def work_per_step(self):
        return 2 * self.M * self.N * self.K

    def host_inputs(self, seed):
        from phew_b200.workloads import normed_matmul_inputs

        return normed_matmul_inputs("typical", seed)

    def setup(self, mx, host):
        base = [mx.array(h) for h in host]
        self.sets = [base] + [[mx.array(a._t.clone()) for a in base] for _ in range(2)]
        self.api(self.sets[0])

    def api(self, inputs):
        from phew_b200.ops import normed_matmul

        return normed_matmul(*inputs, eps=1e-5)

    def launch(self, i):
        self.api(self.sets[i % 3])

    def extras(self, mx):
        from phew_b200.workloads import normed_matmul_fn

        return _opt_over_baseline(self.api, normed_matmul_fn(mx), self.sets[0], self.sets[0])

    def cpu_sample(self, threads: int, rows: int = 1024):
        import numpy as np

        x, w = self.host_inputs(0)
        xs = x[:rows].astype(np.float32)
        wf = w.astype(np.float32)
        t0 = time.perf_counter()
        r = 1.0 / np.sqrt(np.mean(xs.astype(np.float64) ** 2, -1, keepdims=True) + 1e-5)
        _ = (xs @ wf) * r
        dt = time.perf_counter() - t0
        return 2 * rows * self.N * self.K / dt / 1e12, dt, f"{rows} of {self.M} rows (BLAS fp32)"


class RmsNorm:
    """rms_norm fp32 (n, 2048): HBM-bound.  Inputs rotate over enough sets
    that the launches of one timed graph read more than twice the L2."""

    metric, unit, bound, dtype = "rms_norm_hbm_gbs", "GB/s", "hbm", "f32"
    C = 2048
    kernel_regex = "rms_norm"
    SIZES = {256: "small", 1024: "typical", 4096: "large"}

    def __init__(self, n: int = 4096) -> None:
        self.N = n
        self.name = "rms_norm" if n == 4096 else f"rms_norm_n{n}"
        per = self.work_per_step()
        self.R = max(8, -(-2 * L2_BYTES // per) + 1)
        self.min_steps = 2 * self.R  # one graph reads every set twice

    def describe(self):
        return (f"mx.fast.rms_norm fp32 ({self.N},{self.C}), one kernel per step; inputs rotated "
                f"over {self.R} sets ({self.R * self.N * self.C * 4 / 1e6:.0f} MB)")

    def work_per_step(self):
        return 2 * self.N * self.C * 4 + self.C * 4

    def host_inputs(self, seed):
        from phew_b200.workloads import rms_norm_inputs

        return rms_norm_inputs(self.SIZES[self.N], seed)

    def setup(self, mx, host):
        base = [mx.array(h) for h in host]
        self.sets = [base] + [[mx.array(base[0]._t.clone()), base[1]] for _ in range(self.R - 1)]
        self.api(self.sets[0])

    def api(self, inputs):
        from phew_b200 import mx

        return mx.fast.rms_norm(inputs[0], inputs[1], eps=1e-5)

    def launch(self, i):
        self.api(self.sets[i % self.R])

    def extras(self, mx):
        from phew_b200.workloads import rms_norm_fn

        return _opt_over_baseline(self.api, rms_norm_fn(mx), self.sets[0], self.sets[0])

    def cpu_sample(self, threads: int):
        from oracle import mlx_cpu

        x, w = self.host_inputs(0)
        t0 = time.perf_counter()
        mlx_cpu.rms_norm(mlx_cpu.array(x), mlx_cpu.array(w), 1e-5)
        dt = time.perf_counter() - t0
        return self.work_per_step() / dt / 1e9, dt, f"full ({self.N},{self.C})"


L2_BYTES = 126 * 1024 * 1024


def _device_normal(mx, shape, dtype, seed, scale=1.0):
    """A seeded N(0, scale^2) array drawn on the device (phew_fill)."""
    from phew_b200 import _native
    from phew_b200.mx.core import _stream, empty

    out = empty(shape, dtype)
    _native.call("phew_fill", ctypes.c_void_p(out._t.data_ptr()), out.size, shape[-1], out.dtype.code,
                 0, ctypes.c_uint64(seed), ctypes.c_uint64(17), ctypes.c_float(scale), _stream())
    return out


class _DeviceKernelWorkload:
    """A sweep-internal kernel measured on its own, on inputs drawn on the
    device (these arrays are GBs: drawing them on the host would take
    minutes).  The line carries no e2e: these are kernel measurements that
    explain the sweep, not a user-facing call."""

    unit, bound, dtype = "GB/s", "hbm", "bf16"
    e2e = False

    def host_inputs(self, seed):
        return seed

    def launch(self, i):
        self.api(self.sets[i % len(self.sets)])

    def extras(self, mx):
        return {}

    def cpu_sample(self, threads: int):
        return None


class QkvProjection(_DeviceKernelWorkload):
    """The decoder's fused QKV projection at the sweep's typical size:
    x (8 * 2048, 4096) @ W (4096, 12288), bf16, one tcgen05 GEMM per step."""

    name, metric = "qkv_proj", "gemm_tflops"
    unit, bound = "TFLOP/s", "tensor"
    kernel_regex = "gemm_tc"
    profile = "gemm_tc_qkv_proj_bf16_16384x4096x12288"
    M, K, N = 16384, 4096, 12288

    def describe(self):
        return f"x ({self.M},{self.K}) @ W ({self.K},{self.N}) bf16: one tcgen05 GEMM per step"

    def work_per_step(self):
        return 2 * self.M * self.K * self.N

    def setup(self, mx, seed):
        self.sets = [[_device_normal(mx, (self.M, self.K), mx.bfloat16, seed + k),
                      _device_normal(mx, (self.K, self.N), mx.bfloat16, seed + 7, 1.0 / 64.0)]
                     for k in range(2)]
        self.api(self.sets[0])

    def api(self, inputs):
        return inputs[0] @ inputs[1]


class QkScores(_DeviceKernelWorkload):
    """The unfused-attention candidates' score product at seq 8192:
    q (1, 32, 8192, 128) @ k^T, bf16, a batched tcgen05 GEMM with K = 128
    whose (1, 32, 8192, 8192) output makes it bound by HBM writes."""

    name, metric = "qk_scores", "qk_scores_hbm_gbs"
    kernel_regex = "gemm_tc"
    profile = "gemm_tc_qk_scores_bf16_1x32x8192x8192x128"
    B, H, L, D = 1, 32, 8192, 128

    def describe(self):
        return (f"q ({self.B},{self.H},{self.L},{self.D}) @ k^T bf16 -> ({self.B},{self.H},{self.L},{self.L}): "
                "one batched tcgen05 GEMM per step")

    def work_per_step(self):
        # write the scores, read q and k
        return 2 * self.B * self.H * self.L * self.L + 2 * 2 * self.B * self.H * self.L * self.D

    def setup(self, mx, seed):
        shp = (self.B, self.H, self.L, self.D)
        self.sets = [[_device_normal(mx, shp, mx.bfloat16, seed + k),
                      _device_normal(mx, shp, mx.bfloat16, seed + 7)] for k in range(2)]
        self.api(self.sets[0])

    def api(self, inputs):
        return inputs[0] @ inputs[1].transpose(0, 1, 3, 2)


class QkScoresFull(QkScores):
    """The same product at the sweep's full batch: q (8, 32, 8192, 128),
    34 GB of scores per launch."""

    name, metric = "qk_scores_b8", "qk_scores_hbm_gbs"
    profile = None
    B = 8


class Softmax(_DeviceKernelWorkload):
    """mx.softmax over the last axis of bf16 rows 8192 wide (the plain row
    kernel, phew_softmax): the scores of one (8, 32, 8192, 8192) head batch."""

    name, metric = "softmax", "softmax_hbm_gbs"
    kernel_regex = "softmax"
    ROWS, COLS = 262144, 8192

    def describe(self):
        return f"mx.softmax bf16 ({self.ROWS},{self.COLS}) rows, one row kernel per step"

    def work_per_step(self):
        return 2 * self.ROWS * self.COLS * 2

    def setup(self, mx, seed):
        self.sets = [[_device_normal(mx, (self.ROWS, self.COLS), mx.bfloat16, seed, 3.0)]]
        self.api(self.sets[0])

    def api(self, inputs):
        from phew_b200 import mx

        return mx.softmax(inputs[0], axis=-1)


class ScoreSoftmax(_DeviceKernelWorkload):
    """The fused scale + causal-mask + softmax that mx.compile emits for the
    unfused-attention candidates: softmax(s * 1/sqrt(128) + mask) over bf16
    scores (8, 32, 2048, 2048) with an additive (2048, 2048) mask."""

    name, metric = "score_softmax", "score_softmax_hbm_gbs"
    kernel_regex = "softmax"
    profile = "fused_softmax_score_bf16_8x32x2048x2048"
    B, H, L = 8, 32, 2048

    def describe(self):
        return (f"mx.compile'd softmax(s/sqrt(128) + mask) bf16 s ({self.B},{self.H},{self.L},{self.L}), "
                "mask (L, L): one fused row kernel per step")

    def work_per_step(self):
        n = self.B * self.H * self.L * self.L
        return 2 * n * 2 + self.L * self.L * 2

    def setup(self, mx, seed):
        from phew_b200.ops import causal_mask

        self.mask = causal_mask(self.L, self.L, mx.bfloat16)
        self.sets = [[_device_normal(mx, (self.B, self.H, self.L, self.L), mx.bfloat16, seed + k, 10.0)]
                     for k in range(2)]
        scale = 1.0 / math.sqrt(128)

        @mx.compile
        def fn(s, m):
            return mx.softmax(s * scale + m, axis=-1)

        self.fn = fn
        self.api(self.sets[0])

    def api(self, inputs):
        return self.fn(inputs[0], self.mask)


class ScoreSoftmaxLong(ScoreSoftmax):
    """The same fused kernel at seq 8192, where the (8192, 8192) bf16 mask
    (134 MB) no longer fits the L2: s (1, 32, 8192, 8192)."""

    name, metric = "score_softmax_8k", "score_softmax_hbm_gbs"
    profile = "fused_softmax_score_bf16_1x32x8192x8192"
    B, H, L = 1, 32, 8192


class RmsRowMap(_DeviceKernelWorkload):
    """The RMS norm of the decoder block as mx.compile runs it (reduction and
    tail in one row kernel): x * rsqrt(mean(x*x, -1) + 1e-5) * w over bf16
    x (8, 8192, 4096)."""

    name, metric = "rms_rowmap", "rms_rowmap_hbm_gbs"
    kernel_regex = "row_map|phew_rowmap|kernel"
    SHAPE = (8, 8192, 4096)

    def describe(self):
        return f"mx.compile'd x*rsqrt(mean(x*x,-1)+1e-5)*w bf16 x {self.SHAPE}: one row kernel per step"

    def work_per_step(self):
        n = self.SHAPE[0] * self.SHAPE[1] * self.SHAPE[2]
        return 2 * n * 2 + self.SHAPE[2] * 2

    def setup(self, mx, seed):
        self.w = mx.ones((self.SHAPE[2],), mx.bfloat16)
        self.sets = [[_device_normal(mx, self.SHAPE, mx.bfloat16, seed + k)] for k in range(2)]

        @mx.compile
        def fn(x, w):
            return x * mx.rsqrt(mx.mean(x * x, axis=-1, keepdims=True) + 1e-5) * w

        self.fn = fn
        self.api(self.sets[0])

    def api(self, inputs):
        return self.fn(inputs[0], self.w)


WORKLOADS = {
    "gelu_chain": GeluChain,
    "attention": Attention,
    "normed_matmul": NormedMatmul,
    "rms_norm": lambda: RmsNorm(4096),
    "rms_norm_n256": lambda: RmsNorm(256),
    "rms_norm_n1024": lambda: RmsNorm(1024),
    "qkv_proj": QkvProjection,
    "qk_scores": QkScores,
    "qk_scores_b8": QkScoresFull,
    "softmax": Softmax,
    "score_softmax_8k": ScoreSoftmaxLong,
    "score_softmax": ScoreSoftmax,
    "rms_rowmap": RmsRowMap,
}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.workload == "sweep":
        run_reference_sweep(args)
        return
    w = WORKLOADS[args.workload]()
    threads = os.cpu_count() or 1
    if w.cpu_sample(threads) is None:
        # a sweep-internal kernel measured on its own: the reference has no
        # CPU path for it apart from the sweep's (the default workload)
        print(json.dumps({"impl": "reference", "metric": w.metric,
                          "unavailable": f"{args.workload} is a sweep-internal kernel with no CPU "
                                         "counterpart of its own; the reference arm times the sweep"}),
              flush=True)
        return
    for _ in range(max(0, args.warmup - 1)):
        w.cpu_sample(threads)
    vals, secs = [], []
    sample = ""
    for _ in range(args.steps):
        v, dt, sample = w.cpu_sample(threads)
        vals.append(v)
        secs.append(dt)
    val = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": w.metric, "value": val, "unit": w.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(secs) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (np.random.default_rng(0))",
        "config": {"workload": w.describe() + f"; CPU sample {sample} per step"},
        "cpu_baseline": {"value": val, "unit": w.unit, "cores": threads, "kind": "port",
                         "sample": f"{sample} per step, numpy restatement of the MLX-CPU "
                                   f"evaluation on {threads} threads"},
        "e2e": {"value": val, "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's runtime) is not installable here; the oracle port is timed",
    }
    print(json.dumps(line), flush=True)


def measure_kernel(w, mx, d, steps: int, warmup: int, e2e: bool = True) -> dict:
    """Times one workload's kernel: `steps` launches captured in one CUDA
    graph, replayed inside a region bracketed by barrier + synchronize,
    CUDA events on the launching stream, clocks sampled during it; then (if
    `e2e`) the public API with pinned host buffers.  Returns the line's
    fields (value is the whole-job figure over `d.world` replicas)."""
    import numpy as np
    import torch

    from phew_b200 import _native
    from phew_b200.ops import check_device_errors

    dev = mx.core.device()
    stream = torch.cuda.current_stream()
    work = w.work_per_step()
    scale = 1e9 if w.unit == "GB/s" else 1e12
    host = w.host_inputs(d.rank)
    w.setup(mx, host)
    steps = max(steps, getattr(w, "min_steps", 0))

    for i in range(warmup):
        w.launch(i)
    torch.cuda.synchronize()
    # The timed launches are captured once into a CUDA graph, so the timed
    # region measures the device and not the Python host path (which the e2e
    # number below includes).
    graph = torch.cuda.CUDAGraph()
    n0 = _native.launch_count()
    with torch.cuda.graph(graph):
        for i in range(steps):
            w.launch(i)
    graph_launches = _native.launch_count() - n0  # the kernels the timed replay runs
    graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        d.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        d.barrier()
    check_device_errors()
    del graph
    local_ms = ev0.elapsed_time(ev1)
    max_ms = d.max(local_ms)
    value = work * steps * d.world / (max_ms / 1e3) / scale
    achieved = work / (local_ms / steps / 1e3) / scale
    peaks = load_peaks()
    peak = peaks["hbm_gbs"] if w.bound == "hbm" else peaks["bf16_tflops"]
    out = {
        "metric": w.metric, "value": value, "unit": w.unit, "steps": steps,
        "ms_per_step": max_ms / steps, "dtype": w.dtype,
        "workload": w.describe(), "work_per_step": work,
        "roofline": {"bound": w.bound, "achieved": achieved, "peak": peak, "unit": w.unit,
                     "frac": achieved / peak, "traffic": load_traffic(getattr(w, "profile", None)),
                     "peak_source": peaks["source"] + (" (burst)" if w.bound == "tensor" else "")},
        "gpu_launches": graph_launches,
        "clocks": clk.summary(),
    }
    if not e2e or not getattr(w, "e2e", True):
        return out

    # e2e through the public API with pinned host buffers.  Every step
    # copies its inputs host -> device, runs the API call and copies the
    # result device -> host, all inside the timed region; as a streaming
    # caller would, step i + 1's host -> device copy runs on its own stream
    # while step i computes and copies its result back on a third one
    # (inputs double-buffered on the device, events order each buffer's
    # reuse after the compute that read it).
    pinned_in = [torch.from_numpy(np.ascontiguousarray(h.view(np.int16) if h.dtype.itemsize == 2 and h.dtype.kind == "V" else h)).pin_memory()
                 for h in host]
    dev_in = [[torch.empty(p.shape, dtype=a._t.dtype, device=dev) for p, a in zip(pinned_in, w.sets[0])]
              for _ in range(2)]
    out0 = w.api(w.sets[0])
    pinned_out = [torch.empty(out0._t.shape, dtype=out0._t.dtype).pin_memory() for _ in range(2)]
    h2d = sum(p.numel() * p.element_size() for p in pinned_in)
    d2h = pinned_out[0].numel() * pinned_out[0].element_size()
    s_h2d = torch.cuda.Stream(device=dev)
    s_d2h = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # buffer b's inputs have landed
    ev_used = [torch.cuda.Event() for _ in range(2)]  # the compute that read buffer b is done
    used = [False, False]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_h2d):
            if used[b]:
                s_h2d.wait_event(ev_used[b])
            for dst, srcp in zip(dev_in[b], pinned_in):
                dst.view(srcp.dtype).copy_(srcp, non_blocking=True)
            ev_in[b].record(s_h2d)
        stream.wait_event(ev_in[b])
        z = w.api([mx.array(t) for t in dev_in[b]])
        ev_used[b].record(stream)
        used[b] = True
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(ev_used[b])
            z._t.record_stream(s_d2h)
            pinned_out[b].copy_(z._t, non_blocking=True)

    def join_copies():
        for st in (s_h2d, s_d2h):
            e = torch.cuda.Event()
            e.record(st)
            stream.wait_event(e)

    for i in range(2):
        e2e_step(i)
    join_copies()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(steps, 20))
    d.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_h2d.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(i)
    join_copies()
    e1.record(stream)
    torch.cuda.synchronize()
    d.barrier()
    e2e_ms = d.max(e0.elapsed_time(e1))
    out["e2e"] = {"value": work * e2e_steps * d.world / (e2e_ms / 1e3) / scale, "unit": w.unit,
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                  "copies": "every step's H2D and D2H inside the timed region; step i+1's H2D "
                            "overlaps step i's compute and D2H (separate streams)"}
    return out


def run_phew(args) -> None:
    from phew_b200 import mx

    d = Dist()
    w = WORKLOADS[args.workload]()
    m = measure_kernel(w, mx, d, args.steps, args.warmup)
    line = {
        "metric": m["metric"], "value": m["value"], "unit": m["unit"], "n_gpus": d.world,
        "steps": m["steps"], "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": m["dtype"],
        "data": "synthetic (np.random.default_rng(rank))",
        "config": {"workload": m["workload"], "work_per_step": m["work_per_step"],
                   "l2": "inputs larger than L2 or rotated across sets larger than L2",
                   "parallelism": f"replicas x{d.world}"},
        "roofline": m["roofline"], "gpu_launches": m["gpu_launches"], "clocks": m["clocks"],
    }
    if "e2e" in m:
        line["e2e"] = m["e2e"]
    line.update(w.extras(mx))
    if d.rank == 0 and d.world == 1 and not isinstance(w, _DeviceKernelWorkload):
        threads = os.cpu_count() or 1
        v, dt, sample = w.cpu_sample(threads)
        line["cpu_baseline"] = {"value": v, "unit": w.unit, "cores": threads, "kind": "port",
                                "sample": f"{sample}, numpy restatement of the MLX-CPU "
                                          f"evaluation on {threads} threads ({dt * 1e3:.0f} ms)"}
    if d.rank == 0:
        print(json.dumps(line), flush=True)
    d.close()


# ---------------------------------------------------------------------------
# verification sweep (decoder block, 16 candidates)
# ---------------------------------------------------------------------------

SOURCES = ROOT / "tests" / "golden" / "sources"
SIZES = ["small", "typical", "large"]


def decoder_specs(dims, seqs):
    from phew_b200.sweep import ArgSpec
    from phew_b200.workloads import decoder_arg_shapes, decoder_fan_in

    def specs(size):
        shapes = decoder_arg_shapes(seqs[size], dims)
        kinds = ["normal", "ones", "normal", "normal", "normal", "normal", "normal", "causal_mask"]
        return [ArgSpec(tuple(s), "bfloat16", k, f)
                for s, k, f in zip(shapes, kinds, decoder_fan_in(dims))]

    return specs


def _sweep_store(d):
    """The key-value store holding the sweep's shared work counter: the
    process group's store across ranks, an in-process one on one process."""
    from torch.distributed import HashStore

    if not d.dist or d.world == 1:
        return HashStore()
    from torch.distributed import distributed_c10d

    return distributed_c10d._get_default_store()


def _exception_kinds(verdicts) -> dict:
    kinds: dict[str, int] = {}
    for v in verdicts.values():
        for f in v["failures"]:
            if "exception=" in f:
                msg = f.split("exception=", 1)[1]
                k = "out of memory" if "out of memory" in msg else msg.split("(")[0].strip()[:60]
                kinds[k] = kinds.get(k, 0) + 1
    return kinds


def _sweep_setup(args):
    from phew_b200 import sweep
    from phew_b200.workloads import DECODER_FULL, DECODER_SEQ, DECODER_TINY, DECODER_TINY_SEQ

    full = not args.tiny
    dims, seqs = (DECODER_FULL, DECODER_SEQ) if full else (DECODER_TINY, DECODER_TINY_SEQ)
    tag = "decoder_full" if full else "decoder_tiny"
    names = sorted(p.stem for p in SOURCES.glob(f"{tag}__*.py"))
    variants = sweep.VARIANT_SETS[args.variants]
    return dims, seqs, tag, names, variants


def _partial_work(cand: str, failure: str, seq: int, dims) -> tuple[int, int]:
    """(FLOPs, score bytes) a candidate unit did before it raised.  The
    reference's emitted sources raise at a known point: an ``rms_norm`` with
    a full-shape weight (``rms_norm: weight shape``) in the MLP norm, after
    the QKV projection, the attention and the output projection; an SDPA
    output fed to a projection of the wrong width (``matmul: inner
    dimensions differ``) at the output projection, after the QKV projection
    and the attention.  Any other exception counts no work."""
    T, C = dims.batch * seq, dims.dim
    attn = 2 * 2 * dims.batch * dims.heads * seq * seq * dims.head_dim
    sb = 8 * dims.batch * dims.heads * seq * seq if "_sdpa0_" in cand else 0
    msg = failure.split("exception=", 1)[1]
    if msg.startswith("rms_norm: weight shape"):
        return 2 * T * (C * 3 * C + C * C) + attn, sb
    if msg.startswith("matmul: inner dimensions differ"):
        return 2 * T * C * 3 * C + attn, sb
    return 0, 0


def _evaluated_flops(jdir: Path, dims, seqs) -> dict:
    """Algorithmic work of a sweep, from its journals: every group's
    baseline, each candidate that ran to a comparison, and the part of each
    raising candidate that ran before it raised (`_partial_work`).

    Score bytes: a graph that computes attention unfused (the baseline and
    the candidates without the SDPA substitution, ``sdpa0`` in their names)
    writes the (batch, heads, seq, seq) bf16 scores once (QK^T), reads them
    and writes P once (the fused scale + mask + softmax) and reads P once
    (P V): 8 bytes per score."""
    from phew_b200 import sweep
    from phew_b200.workloads import decoder_flops

    w = {"flops": 0, "score_bytes": 0, "partial_flops": 0, "partial_score_bytes": 0,
         "evaluated": 0, "raised": 0}
    for p in sorted(jdir.glob("journal.rank*.jsonl")):
        for g in sweep.load_groups(p).values():
            seq = seqs[g.size]
            f = decoder_flops(seq, dims)
            sb = 8 * dims.batch * dims.heads * seq * seq
            # the baseline (unfused attention) ran unless every unit of the group raised
            if any(r is None or "exception=" not in r for r in g.results.values()):
                w["flops"] += f
                w["score_bytes"] += sb
            for cand, r in g.results.items():
                if r is not None and "exception=" in r:
                    w["raised"] += 1
                    pf, pb = _partial_work(cand, r, seq, dims)
                    w["partial_flops"] += pf
                    w["partial_score_bytes"] += pb
                else:
                    w["evaluated"] += 1
                    w["flops"] += f
                    if "_sdpa0_" in cand:
                        w["score_bytes"] += sb
    return w


# Groups whose host-drawn inputs are prepared ahead of the one being
# evaluated in the e2e sweep (pinned buffers: depth + 1 sets).
E2E_DEPTH = 2


def _timed_sweep(d, groups, names, ev, store, journal, run_id, prefetch=None, prefetch_depth=1):
    """One sweep over `groups` inside a region bracketed by barrier +
    synchronize; returns (device seconds on this rank, wall seconds,
    library launches, clocks)."""
    import torch

    from phew_b200 import _native, sweep

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        d.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        n0 = _native.launch_count()
        e0.record()
        sweep.run_groups(groups, names, ev, store, d.rank, journal=journal, run_id=run_id,
                         prefetch=prefetch, prefetch_depth=prefetch_depth)
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        launches = _native.launch_count() - n0
        d.barrier()
    return e0.elapsed_time(e1) / 1e3, wall, launches, clk.summary()


def _shared_dir(d, prefix: str, given: str | None) -> Path:
    jdir = Path(given) if given else Path(tempfile.mkdtemp(prefix=prefix))
    if d.dist:  # every rank journals into rank 0's directory
        obj = [str(jdir)]
        d.dist.broadcast_object_list(obj, src=0)
        jdir = Path(obj[0])
    jdir.mkdir(parents=True, exist_ok=True)
    return jdir


def _host_threads(d) -> int:
    """Host threads one rank may use for input draws: the cores this
    process may run on, shared by the ranks of the node, one left for the
    thread that launches kernels."""
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    local = int(os.environ.get("LOCAL_WORLD_SIZE", str(d.world)))
    return max(1, cores // max(1, local) - 1)


def run_sweep(args) -> None:
    import torch

    from phew_b200 import mx, sweep
    from phew_b200.ops import check_device_errors
    from phew_b200.verify import checker as checker_mod
    from phew_b200.workloads import decoder_block_fn, decoder_flops

    d = Dist()
    mx.core.device()
    dims, seqs, tag, names, variants = _sweep_setup(args)
    cands = sweep.load_candidates({n: (SOURCES / f"{n}.py").read_text() for n in names})
    baseline = decoder_block_fn(mx, dims)
    seeds = list(range(args.seeds))
    shards = sweep.make_shards(names, seeds)
    groups = sweep.make_groups(seeds, SIZES, variants)
    store = _sweep_store(d)
    specs = decoder_specs(dims, seqs)
    ev = sweep.DeviceEvaluator(baseline, cands, sweep.DeviceInputs(specs))

    # warm-up (untimed): W passes of every candidate at one size, sizes
    # cycling large -> small, so every size's runtime-compiled kernels are
    # built (each size compiles its own) before the timed region
    order = list(reversed(SIZES))
    for i in range(max(args.warmup, len(SIZES))):
        for c in names:
            ev(c, 99, order[i % len(order)], variants[0])
    ev.release()
    torch.cuda.synchronize()

    jdir = _shared_dir(d, "sweep_", args.journal_dir)
    dev_s, wall, launches, clocks = _timed_sweep(
        d, groups, names, ev, store, jdir / f"journal.rank{d.rank}.jsonl", f"sweep/{jdir.name}")
    check_device_errors()
    max_s = d.max(dev_s)
    max_wall = d.max(wall)
    ev.release()

    # e2e: the same sweep with inputs drawn on the host and copied in
    e2e = None
    if not args.no_e2e and args.variants == "edge":
        host_in = sweep.HostInputs(specs, SIZES, threads=_host_threads(d), slots=E2E_DEPTH + 1)
        ev2 = sweep.DeviceEvaluator(baseline, cands, host_in)
        rb0 = checker_mod.readback_bytes
        edir = _shared_dir(d, "sweep_e2e_", None)
        e2e_s, e2e_wall, _, e2e_clocks = _timed_sweep(
            d, groups, names, ev2, store, edir / f"journal.rank{d.rank}.jsonl",
            f"sweep_e2e/{edir.name}", prefetch=host_in.prefetch, prefetch_depth=E2E_DEPTH)
        check_device_errors()
        host_in.close()
        ev2.release()
        h2d = d.sum(host_in.h2d_bytes)
        d2h = d.sum(checker_mod.readback_bytes - rb0)
        e2e_max = d.max(e2e_s)
        e2e = {"value": len(names) / e2e_max, "unit": "candidates/s", "seconds": e2e_max,
               "h2d_bytes_per_step": h2d / args.steps, "d2h_bytes_per_step": d2h / args.steps,
               "h2d_bytes_total": h2d, "d2h_bytes_total": d2h,
               "copies": "every group's 8 arguments drawn on the host (phew_fill_host, "
                         f"{_host_threads(d)} threads per rank, up to {E2E_DEPTH} groups ahead on a "
                         "background thread, pinned) and copied host -> device; every comparison "
                         "record copied device -> host; all inside the timed region",
               "clocks": e2e_clocks, "journal": str(edir)}
        del host_in
    torch.cuda.empty_cache()

    line = None
    if d.rank == 0:
        verdicts, missing = sweep.merge(jdir, shards, SIZES, variants)
        units = len(shards) * len(SIZES) * len(variants)
        work = _evaluated_flops(jdir, dims, seqs)
        flops, evaluated, raised = work["flops"], work["evaluated"], work["raised"]
        peaks = load_peaks()
        achieved = flops / d.world / max_s / 1e12
        peak = peaks["bf16_tflops_sustained"]
        # the time the sweep's work needs at the measured peaks: its FLOPs
        # (raising units' partial work included) at the sustained GEMM rate
        # plus the unfused graphs' score traffic at the HBM copy rate
        # (separate kernels, so the two add)
        all_flops = flops + work["partial_flops"]
        score_bytes = work["score_bytes"] + work["partial_score_bytes"]
        flop_s = all_flops / d.world / (peak * 1e12)
        byte_s = score_bytes / d.world / (peaks["hbm_gbs"] * 1e9)
        line = {
            "metric": "verified_candidates_per_s", "value": len(names) / max_s,
            "unit": "candidates/s", "n_gpus": d.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_s * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (counter-based generator; device draws for value, host draws for e2e)",
            "config": {
                "workload": f"{tag} verification sweep: {len(names)} candidates x {len(seeds)} seeds x "
                            f"seq {[seqs[z] for z in SIZES]} x variants {list(variants)}",
                "dims": dict(batch=dims.batch, dim=dims.dim, heads=dims.heads, hidden=dims.hidden),
                "step": f"1/{args.steps} of one full sweep: the timed region is the whole sweep "
                        f"({len(groups)} groups); ms_per_step = region / steps",
                "warmup": f"{max(args.warmup, len(SIZES))} untimed passes of every candidate at one "
                          "size (sizes cycling large -> small; builds every runtime-compiled kernel)",
                "l2": "every group's inputs (>= 520 MB) exceed the L2",
                "parallelism": f"(seed, size, variant) groups over {d.world} rank(s) from one "
                               "host-side counter, no data-path collective"},
            "units_per_s": units / max_s, "units": units, "evaluated_units": evaluated,
            "raising_units": raised,
            "evaluated_tflop": flops / 1e12,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None,
                         "kernel": "the whole sweep: algorithmic FLOPs of every baseline and every "
                                   "candidate unit that ran to a comparison, per GPU-second",
                         "peak_source": peaks["source"] + " (sustained)"},
            "roofline_model": {
                "ideal_s": flop_s + byte_s, "frac": (flop_s + byte_s) / max_s,
                "flop_s": flop_s, "score_byte_s": byte_s,
                "tflop": all_flops / 1e12, "partial_tflop": work["partial_flops"] / 1e12,
                "score_gb": score_bytes / 1e9,
                "model": "per GPU: FLOPs of every unit (the raising units' work up to the op "
                         "that raised included) / sustained bf16 peak + bytes of the (batch, "
                         "heads, seq, seq) score tensor the unfused-attention graphs write and "
                         "read (8 B per score) / HBM copy peak"},
            "wall_s": max_wall,
            "passed": sorted(c for c, v in verdicts.items() if v["passed"]),
            "failed": sorted(c for c, v in verdicts.items() if not v["passed"]),
            "missing_shards": len(missing),
            # units that failed by raising, by kind (a device out-of-memory here
            # would be a backend fault, not a verdict)
            "exception_units": _exception_kinds(verdicts),
            "clocks": clocks, "journal": str(jdir),
            "gpu_launches": launches,  # rank 0's; every rank launches its own groups' kernels
        }
        if e2e is not None:
            e2e_verdicts, _ = sweep.merge(Path(e2e["journal"]), shards, SIZES, variants)
            e2e["verdicts_match"] = {c: v["passed"] for c, v in e2e_verdicts.items()} == \
                {c: v["passed"] for c, v in verdicts.items()}
            line["e2e"] = e2e

    if d.world == 1:
        # GPU units/s on the CPU subset (seed 0, the small size, 4 variants)
        sub = [sweep.Group(0, "small", v) for v in variants]
        sub_s, _, _, _ = _timed_sweep(d, sub, names, ev, _sweep_store(d), None, "subset")
        ev.release()
        line["gpu_units_per_s_subset"] = len(sub) * len(names) / sub_s
        if not args.no_configs and not args.tiny:
            line["configs"] = measure_configs(mx, d, args)
        threads = os.cpu_count() or 1
        cb = cpu_sweep_sample(args, args.cpu_units, 0, threads)
        line["cpu_baseline"] = {"value": cb["value"], "unit": "candidates/s", "cores": threads,
                                "kind": "port", "sample": cb["sample"],
                                "units_per_s_subset": cb["units_per_s_subset"]}
    if d.rank == 0:
        print(json.dumps(line), flush=True)
    _ = decoder_flops
    d.close()


def measure_configs(mx, d, args) -> dict:
    """Per-kernel figures of benchmark configs 0-3 on this GPU (value,
    roofline fraction, clocks, optimized/baseline ms)."""
    import torch

    out = {}
    for name in ("rms_norm_n256", "rms_norm_n1024", "rms_norm", "gelu_chain", "attention",
                 "normed_matmul"):
        w = WORKLOADS[name]()
        m = measure_kernel(w, mx, d, args.steps, args.warmup, e2e=False)
        ex = w.extras(mx)
        out[name if name != "rms_norm" else "rms_norm_n4096"] = {
            "metric": m["metric"], "value": m["value"], "unit": m["unit"],
            "frac": m["roofline"]["frac"], "peak": m["roofline"]["peak"],
            "peak_source": m["roofline"]["peak_source"], "traffic": m["roofline"]["traffic"],
            "ms_per_launch": m["ms_per_step"], "launches": m["steps"], "workload": m["workload"],
            "clocks": m["clocks"], **ex}
        del w
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# the sweep on the CPU (oracle), on the 64-unit subset
# ---------------------------------------------------------------------------


def _oracle_candidates(names):
    from oracle import mlx_cpu

    mlx_cpu.CUDA_CHAINS.update(json.loads((SOURCES / "cuda_chains.json").read_text()))
    out = {}
    for name in names:
        src = (SOURCES / f"{name}.py").read_text()
        src = src.replace("import phew_b200.mx as mx", "import oracle.mlx_cpu as mx")
        src = src.replace("from phew_b200.mx import fast", "from oracle.mlx_cpu import fast")
        ns: dict = {}
        exec(compile(src, name, "exec"), ns)
        out[name] = ns["optimized"]
    return out


def _cpu_variant_inputs(specs, variant: str, seed: int, batch_rows: int, threads: int):
    """One edge variant's arguments for the CPU sample, drawn on the host
    with numpy (independent generators per chunk, on `threads` threads):
    x keeps `batch_rows` of its batch rows, the weights are full size."""
    import zlib

    import numpy as np

    from oracle import mlx_cpu

    out = []
    ss = np.random.SeedSequence([seed, zlib.crc32(variant.encode())])  # stable across processes
    for i, spec in enumerate(specs):
        shape = list(spec.shape)
        if i == 0:
            shape[0] = batch_rows
        n = int(np.prod(shape))
        a = np.zeros(n, np.float32)
        if variant in ("pm1e4", "subnormal"):
            scale = 1e4 if variant == "pm1e4" else 1e-39
            kids = ss.spawn(threads)
            per = -(-n // threads)

            def draw(t):
                lo, hi = t * per, min(n, (t + 1) * per)
                if lo < hi:
                    np.random.default_rng(kids[t]).standard_normal(hi - lo, dtype=np.float32,
                                                                   out=a[lo:hi])
            with cf.ThreadPoolExecutor(max_workers=threads) as ex:
                list(ex.map(draw, range(threads)))
            a *= np.float32(scale)
        elif variant == "one_hot_rows":
            rows = a.reshape(-1, shape[-1])
            hot = np.random.default_rng(ss).integers(0, shape[-1], rows.shape[0])
            rows[np.arange(rows.shape[0]), hot] = 1.0
        elif variant != "zeros":
            raise ValueError(f"CPU sample: variant {variant!r}")
        out.append(mlx_cpu.array(a.reshape(shape).astype(mlx_cpu.BF16)))
    return out


def cpu_sweep_sample(args, n_units: int, first_unit: int, threads: int) -> dict:
    """Times the oracle on units of the 64-unit subset (16 candidates x
    seed 0 x the small size x 4 variants, variant-major), each on
    `batch_rows` of the decoder's batch rows; a variant's baseline is
    evaluated (and timed) with its first unit.  Returns the units/s on the
    subset (in full units: the batch slice is 1/batch of a unit) and the
    candidates/s it implies for the full sweep, by the algorithmic FLOPs of
    each size relative to the sampled one."""
    import numpy as np

    from oracle import mlx_cpu, verdict
    from phew_b200.workloads import decoder_block_fn, decoder_flops

    dims, seqs, tag, names, variants = _sweep_setup(args)
    specs = decoder_specs(dims, seqs)("small")
    ocands = _oracle_candidates(names)
    base_fn = decoder_block_fn(mlx_cpu, dims)
    tol = verdict.checker_tolerance({"fp32_to_fp32"})
    batch_rows = 1
    frac = batch_rows / dims.batch
    cache: dict[str, tuple] = {}
    secs = 0.0
    for u in range(first_unit, first_unit + n_units):
        v = variants[(u // len(names)) % len(variants)]
        c = names[u % len(names)]
        if v not in cache:
            host = _cpu_variant_inputs(specs, v, 0, batch_rows, threads)  # untimed draw
            t0 = time.perf_counter()
            try:
                b = base_fn(*host)
            except Exception:  # noqa: BLE001
                b = None
            secs += time.perf_counter() - t0
            cache.clear()
            cache[v] = (host, b)
        host, b = cache[v]
        t0 = time.perf_counter()
        try:
            co = ocands[c](*host)
            if b is not None:
                bn = np.asarray(b).astype(np.float32)
                cn = np.asarray(co).astype(np.float32)
                verdict.compare_output(bn, cn, tol, True)
        except Exception:  # noqa: BLE001  (a raising unit is a failed unit)
            pass
        secs += time.perf_counter() - t0
    units_per_s = n_units * frac / secs
    # one candidate of the full sweep: |seeds| x |variants| units at each size
    rel = sum(decoder_flops(seqs[z], dims) for z in SIZES) / decoder_flops(seqs["small"], dims)
    per_candidate_s = args.seeds * len(variants) * rel / units_per_s
    return {"value": 1.0 / per_candidate_s, "units_per_s_subset": units_per_s, "seconds": secs,
            "sample": f"{n_units} unit(s) of the 64-unit subset (16 candidates x seed 0 x seq "
                      f"{seqs['small']} x 4 variants), each on {batch_rows} of {dims.batch} batch "
                      f"rows, baselines included; numpy restatement of the MLX-CPU evaluation on "
                      f"{threads} threads; candidates/s of the full sweep extrapolated by "
                      f"algorithmic FLOPs per size ({secs:.1f} s)"}


def run_reference_sweep(args) -> None:
    """The reference arm for the sweep: the oracle port on the host CPU, a
    step = one unit of the 64-unit subset (on one batch row), all host
    threads."""
    threads = os.cpu_count() or 1
    warm = cpu_sweep_sample(args, args.warmup, 0, threads) if args.warmup else None
    res = cpu_sweep_sample(args, args.steps, args.warmup, threads)
    _ = warm
    line = {
        "impl": "reference", "metric": "verified_candidates_per_s", "value": res["value"],
        "unit": "candidates/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds"] * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (numpy default_rng, host)",
        "config": {"workload": "decoder-block verification sweep on the CPU; a step = one unit of "
                               "the 64-unit subset on one batch row"},
        "units_per_s_subset": res["units_per_s_subset"],
        "cpu_baseline": {"value": res["value"], "unit": "candidates/s", "cores": threads,
                         "kind": "port", "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": "candidates/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's runtime) is not installable here; the oracle port is timed",
    }
    print(json.dumps(line), flush=True)


def main(argv=None) -> int:
    args = parse_args(sys.argv[1:] if argv is None else argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "sweep":
        run_sweep(args)
    else:
        run_phew(args)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
