"""Benchmark of phew's candidate-evaluation path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl phew|reference]
                    [--workload gelu_chain|attention|normed_matmul|rms_norm]

Default workload (gelu_chain): the fused elementwise chain
z = tanh-GELU(x*a + b) * sigmoid(c) + x on fp16 (4096, 8192) -- the
fuse->=3-ops path, HBM-bound.  A step is one launch of the fused kernel over
one batch of inputs.  The other workloads time one launch of the attention
kernel (bf16 (4, 32, 2048, 128), causal), the normed matmul
(x bf16 (8192, 4096) @ W (4096, 4096), fused row norm) and rms_norm
(fp32 (4096, 2048)).

Printed (one JSON line, rank 0):
  value       the workload's throughput over all ranks (HBM GB/s for the
              memory-bound kernels, TFLOP/s for the tensor-core ones) with
              inputs resident in HBM and rotated so no step finds its inputs in
              the 126 MB L2
  e2e         the same metric through the public API with pinned host
              buffers: H2D of the inputs and D2H of the output inside every
              step (step i+1's H2D overlapping step i's compute and D2H)
  roofline    achieved vs the measured HBM copy bandwidth / cuBLAS bf16 peak
  cpu_baseline  the oracle (numpy restatement of the MLX-CPU evaluation)
              timed on a bounded sample on the host
  optimized_ms / baseline_ms   (gelu_chain) fused kernel vs the unfused
              op-by-op evaluation of the same harness function on this backend

``--impl reference`` times the reference's path on the host CPU (the oracle
port: MLX, the reference's runtime, is not installable here), using all
host threads, on the same workload and metric.

Multi-GPU (torchrun): every rank runs its own replica (weak scaling); the
timed region is bracketed by a barrier and device synchronisation, and the
max time over ranks is reported.
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
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["phew", "reference"], default="phew")
    ap.add_argument("--workload", default="gelu_chain",
                    choices=["gelu_chain", "attention", "normed_matmul", "rms_norm"])
    return ap.parse_args(argv)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


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
    """rms_norm fp32 (4096, 2048): HBM-bound (inputs rotated past the L2)."""

    name = "rms_norm"
    metric, unit, bound, dtype = "rms_norm_hbm_gbs", "GB/s", "hbm", "f32"
    N, C = 4096, 2048
    kernel_regex = "rms_norm"
    R = 8

    def describe(self):
        return f"mx.fast.rms_norm fp32 ({self.N},{self.C}), one kernel per step"

    def work_per_step(self):
        return 2 * self.N * self.C * 4 + self.C * 4

    def host_inputs(self, seed):
        from phew_b200.workloads import rms_norm_inputs

        return rms_norm_inputs("large", seed)

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


WORKLOADS = {c.name: c for c in (GeluChain, Attention, NormedMatmul, RmsNorm)}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    w = WORKLOADS[args.workload]()
    threads = os.cpu_count() or 1
    for _ in range(max(1, args.warmup)):
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


def run_phew(args) -> None:
    import numpy as np
    import torch

    from phew_b200 import mx
    from phew_b200.ops import check_device_errors

    d = Dist()
    dev = mx.core.device()
    stream = torch.cuda.current_stream()
    w = WORKLOADS[args.workload]()
    work = w.work_per_step()
    scale = 1e9 if w.unit == "GB/s" else 1e12
    host = w.host_inputs(d.rank)
    w.setup(mx, host)

    for i in range(args.warmup):
        w.launch(i)
    torch.cuda.synchronize()
    # The K timed launches are captured once into a CUDA graph, so the timed
    # region measures the device and not the Python host path (which the e2e
    # number below includes).
    from phew_b200 import _native

    graph = torch.cuda.CUDAGraph()
    n0 = _native.launch_count()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
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
    value = work * args.steps * d.world / (max_ms / 1e3) / scale
    achieved = work / (local_ms / args.steps / 1e3) / scale

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
    e2e_steps = max(3, min(args.steps, 20))
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
    e2e_val = work * e2e_steps * d.world / (e2e_ms / 1e3) / scale

    peaks = load_peaks()
    peak = peaks["hbm_gbs"] if w.bound == "hbm" else peaks["bf16_tflops"]
    line = {
        "metric": w.metric, "value": value, "unit": w.unit, "n_gpus": d.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (np.random.default_rng(rank))",
        "config": {"workload": w.describe(), "work_per_step": work,
                   "l2": "inputs larger than L2 or rotated across sets larger than L2",
                   "parallelism": f"replicas x{d.world}"},
        "roofline": {"bound": w.bound, "achieved": achieved, "peak": peak, "unit": w.unit,
                     "frac": achieved / peak, "traffic": load_traffic(getattr(w, "profile", None)),
                     "peak_source": peaks["source"] + (" (burst)" if w.bound == "tensor" else "")},
        "e2e": {"value": e2e_val, "unit": w.unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "copies": "every step's H2D and D2H inside the timed region; step i+1's H2D "
                          "overlaps step i's compute and D2H (separate streams)"},
        "gpu_launches": graph_launches,
        "clocks": clk.summary(),
    }
    line.update(w.extras(mx))
    if d.rank == 0 and d.world == 1:
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


def run_sweep(args) -> None:
    import torch

    from phew_b200 import _native, mx, sweep
    from phew_b200.ops import check_device_errors
    from phew_b200.workloads import DECODER_FULL, DECODER_SEQ, DECODER_TINY, DECODER_TINY_SEQ, decoder_block_fn

    d = Dist()
    mx.core.device()
    full = not args.tiny
    dims, seqs = (DECODER_FULL, DECODER_SEQ) if full else (DECODER_TINY, DECODER_TINY_SEQ)
    tag = "decoder_full" if full else "decoder_tiny"
    names = sorted(p.stem for p in SOURCES.glob(f"{tag}__*.py"))
    cands = sweep.load_candidates({n: (SOURCES / f"{n}.py").read_text() for n in names})
    baseline = decoder_block_fn(mx, dims)
    seeds = list(range(args.seeds))
    sizes = ["small", "typical", "large"]
    variants = sweep.VARIANT_SETS[args.variants]
    shards = sweep.make_shards(names, seeds)
    groups = sweep.make_groups(seeds, sizes, variants)
    store = _sweep_store(d)
    jdir = Path(args.journal_dir) if args.journal_dir else Path(tempfile.mkdtemp(prefix="sweep_"))
    if d.dist:  # every rank journals into rank 0's directory
        obj = [str(jdir)]
        d.dist.broadcast_object_list(obj, src=0)
        jdir = Path(obj[0])
    jdir.mkdir(parents=True, exist_ok=True)
    journal = jdir / f"journal.rank{d.rank}.jsonl"
    ev = sweep.DeviceEvaluator(baseline, cands, sweep.DeviceInputs(decoder_specs(dims, seqs)))

    # warm-up: compile every kernel the candidates use (generated kernels
    # specialise on row length, so each size compiles its own), untimed
    for size in sizes:
        for c in names:
            ev(c, 99, size, variants[0])
    ev.release()
    torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        d.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        n0 = _native.launch_count()
        e0.record()
        recs = sweep.run_groups(groups, names, ev, store, d.rank, journal=journal,
                                run_id=f"sweep/{jdir.name}")
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        launches = _native.launch_count() - n0
        d.barrier()
    check_device_errors()
    dev_s = e0.elapsed_time(e1) / 1e3
    max_s = d.max(dev_s)
    max_wall = d.max(wall)
    if d.rank == 0:
        verdicts, missing = sweep.merge(jdir, shards, sizes, variants)
        units = len(shards) * len(sizes) * len(variants)
        line = {
            "metric": "verified_candidates_per_s", "value": len(names) / max_s,
            "unit": "candidates/s", "n_gpus": d.world, "steps": 1, "warmup": 1,
            "ms_per_step": max_s * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (device counter-based RNG)",
            "config": {"workload": f"{tag} verification sweep: {len(names)} candidates x {len(seeds)} "
                                   f"seeds x sizes {[seqs[s] for s in sizes]} x variants {list(variants)}",
                       "dims": vars(dims) if hasattr(dims, "__dict__") else str(dims),
                       "warmup": "each candidate once at every size (runtime kernel compilation)",
                       "parallelism": f"(seed, size, variant) groups over {d.world} rank(s) from one "
                                      "host-side counter, no data-path collective"},
            "units_per_s": units / max_s, "units": units, "wall_s": max_wall,
            "passed": sorted(c for c, v in verdicts.items() if v["passed"]),
            "failed": sorted(c for c, v in verdicts.items() if not v["passed"]),
            "missing_shards": len(missing),
            # units that failed by raising, by kind (a device out-of-memory here
            # would be a backend fault, not a verdict)
            "exception_units": _exception_kinds(verdicts),
            "clocks": clk.summary(), "journal": str(jdir),
            "gpu_launches": launches,  # rank 0's; every rank launches its own groups' kernels
        }
        print(json.dumps(line), flush=True)
    _ = recs
    d.close()


def main(argv=None) -> int:
    if argv is None:
        argv = sys.argv[1:]
    if "--workload" in argv and "sweep" in argv:
        ap = argparse.ArgumentParser()
        ap.add_argument("--gpus", type=int, default=1)
        ap.add_argument("--steps", type=int, default=1)
        ap.add_argument("--warmup", type=int, default=1)
        ap.add_argument("--impl", default="phew")
        ap.add_argument("--workload", default="sweep")
        ap.add_argument("--seeds", type=int, default=5)
        ap.add_argument("--variants", choices=["edge", "reference"], default="edge")
        ap.add_argument("--tiny", action="store_true")
        ap.add_argument("--journal-dir", default=None)
        run_sweep(ap.parse_args(argv))
        return 0
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_phew(args)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
