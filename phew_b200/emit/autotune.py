"""Phase-2 launch-parameter search for runtime-compiled CUDA kernels.

Stands in for ``KernelParamSearch`` (phew ``emit/metal_kernel.py:59-270``),
which ``Optimizer.run`` step 5a (``optimizer.py:250-279``) runs on kernel
nodes the passes did not replace.  Same interface and flow:

1. enumerate parameterisations, filtered by the bottleneck class the
   profile step produced (``_apply_bottleneck_filter``, same rules);
2. prune with the cost model's hard limits (``cost/pruner.py:23-48``:
   block size over the device limit) and the B200's shared-memory limit;
3. time the survivors with CUDA events (``phew_b200.bench.benchmark``, cold
   L2) on the "typical" inputs;
4. verify the five fastest against the baseline function
   (``phew_b200.verify.EquivalenceChecker``, every seed and variant, at the
   traced shapes the kernel's outputs are declared with) and return the
   verified ones, fastest first.

Knobs on B200: the block size (threadgroup) and, for grid-stride kernels,
the grid as waves of resident threads per SM (the emitted chains loop over
their elements, so the grid is free); the template constants ``VW``
(vector width) and ``UNROLL`` reach the kernel only when its source names
them, exactly as the reference injects them.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

THREADGROUP_1D = [64, 128, 256, 512, 1024]
WAVES = [1, 2, 4, 8, 16]          # grid = waves x resident threads of the device
VECTOR_WIDTHS = [1, 2, 4, 8]
LOOP_UNROLLS = [1, 2, 4, 8]
MAX_THREADS_PER_BLOCK = 1024
MAX_THREADS_PER_SM = 2048
MAX_SMEM_PER_BLOCK = 227 * 1024


@dataclass
class KernelCandidate:
    """One parameterisation of a kernel (field names of the reference's)."""

    threadgroup: tuple[int, ...]
    tile: tuple[int, int] | None
    vector_width: int
    loop_unroll: int
    use_threadgroup_mem: bool
    use_constant_address: bool
    template_params: list[tuple[str, object]] = field(default_factory=list)
    source: str = ""
    measured_ms: float | None = None
    verified: bool = False
    pruned: bool = False
    prune_reason: str = ""
    waves: int = 8
    grid: tuple[int, int, int] | None = None
    source_uses_vw: bool = False
    source_uses_unroll: bool = False


class KernelParamSearch:
    """Phase-2 parameter search for a hot kernel on this backend."""

    def __init__(self, baseline_fn: Callable | None = None, max_candidates: int = 50,
                 bottleneck: Any = None) -> None:
        self.baseline_fn = baseline_fn
        self.max_candidates = max_candidates
        self.bottleneck = bottleneck

    # -- search --------------------------------------------------------------

    def search(self, kernel_node: Any, input_factory: Callable[[str, int], tuple[list, dict]],
               profile_data: Any = None) -> list[KernelCandidate]:
        from ..bench import benchmark
        from ..verify import EquivalenceChecker

        surviving = []
        for cand in self._enumerate(kernel_node):
            prune, reason = self._prune(kernel_node, cand)
            if prune:
                cand.pruned, cand.prune_reason = True, reason
            else:
                surviving.append(cand)
        surviving = surviving[: self.max_candidates]

        args, kwargs = input_factory("typical", 0)
        for cand in surviving:
            try:
                fn = self._build_kernel_fn(kernel_node, cand)
                cand.measured_ms = benchmark(fn, *args, n_warmup=3, n_bench=10, **kwargs).mean_ms
            except Exception as exc:  # noqa: BLE001  (a failing candidate is pruned)
                cand.pruned, cand.prune_reason = True, str(exc)

        measured = sorted((c for c in surviving if c.measured_ms is not None),
                          key=lambda c: c.measured_ms)
        checker = EquivalenceChecker()
        # The kernel's output shapes are those it was traced at, so every
        # verification size runs the traced ("typical") shapes: a kernel
        # without a launch contract must never see larger inputs than the
        # outputs it writes.
        typical = lambda size, seed: input_factory("typical", seed)  # noqa: E731
        for cand in measured[:5]:
            if self.baseline_fn is None:
                cand.verified = True
                continue
            res = checker.check(self.baseline_fn, self._build_kernel_fn(kernel_node, cand), typical)
            cand.verified = res.passed
        return [c for c in measured if c.verified]

    # -- enumeration -----------------------------------------------------------

    def _enumerate(self, node: Any) -> list[KernelCandidate]:
        all_c = list(self._enumerate_all(node))
        kept = list(self._apply_bottleneck_filter(all_c))
        return kept if kept else all_c

    def _enumerate_all(self, node: Any):
        src = getattr(node, "source", "") or ""
        vws = VECTOR_WIDTHS if "VW" in src else [1]
        unrolls = LOOP_UNROLLS if "UNROLL" in src else [1]
        waves_set = WAVES if self.grid_stride(node) else [0]
        for tg in THREADGROUP_1D:
            for waves in waves_set:
                for vw in vws:
                    for unroll in unrolls:
                        yield KernelCandidate(
                            threadgroup=(tg,), tile=None, vector_width=vw, loop_unroll=unroll,
                            use_threadgroup_mem=False, use_constant_address=False,
                            template_params=[("THREADGROUP", tg), ("VW", vw), ("UNROLL", unroll)],
                            waves=waves, source_uses_vw="VW" in src, source_uses_unroll="UNROLL" in src,
                        )

    def _apply_bottleneck_filter(self, candidates: list[KernelCandidate]):
        """The reference's routing by bottleneck class (metal_kernel.py:186-228):
        memory-bound keeps wide vectors and blocks >= 128, compute-bound keeps
        warp-multiple blocks, launch-overhead keeps blocks >= 256 with deep
        unrolls, occupancy-limited keeps blocks <= 128.  A knob the source
        does not use does not filter."""
        bn = getattr(self.bottleneck, "value", self.bottleneck)
        for c in candidates:
            tg = c.threadgroup[0]
            uses_vw, uses_unroll = c.source_uses_vw, c.source_uses_unroll
            if bn == "memory_bound" and not (tg >= 128 and (c.vector_width >= 2 or not uses_vw)):
                continue
            if bn == "compute_bound" and tg % 32:
                continue
            if bn == "launch_overhead" and not (tg >= 256 and (c.loop_unroll >= 4 or not uses_unroll)):
                continue
            if bn == "occupancy_limited" and tg > 128:
                continue
            yield c

    # -- pruning -----------------------------------------------------------------

    def _prune(self, node: Any, cand: KernelCandidate) -> tuple[bool, str]:
        tg = cand.threadgroup[0] * (cand.threadgroup[1] if len(cand.threadgroup) > 1 else 1)
        if tg > MAX_THREADS_PER_BLOCK:
            return True, f"threadgroup_size={tg} > {MAX_THREADS_PER_BLOCK}"
        smem = int(getattr(node, "attrs", {}).get("threadgroup_mem_bytes", 0) or 0)
        if smem > MAX_SMEM_PER_BLOCK:
            return True, f"threadgroup_mem={smem}B > limit={MAX_SMEM_PER_BLOCK}B"
        return False, ""

    # -- execution -----------------------------------------------------------------

    @staticmethod
    def grid_stride(node: Any) -> bool:
        """Kernels this backend emits loop over their elements with a grid
        stride (``phew_nthreads``), so any grid covers them; a user kernel
        keeps the grid it was written for."""
        return "phew_nthreads" in (getattr(node, "source", "") or "")

    def _grid(self, node: Any, cand: KernelCandidate, inputs) -> tuple[int, int, int]:
        from ..mx.core import sm_count

        n = inputs[0].size if inputs else 1
        g = getattr(node, "grid", None)
        if not self.grid_stride(node):
            g = g if g is not None else (n, 1, 1)
            return tuple(int(v) for v in (tuple(g) + (1, 1, 1))[:3])
        resident = sm_count() * MAX_THREADS_PER_SM
        threads = min(max(int(n), 1), cand.waves * resident)
        return (max(threads, cand.threadgroup[0]), 1, 1)

    def _build_kernel_fn(self, node: Any, cand: KernelCandidate) -> Callable:
        from .. import dtypes as dt
        from ..mx.fast import cuda_kernel

        source = getattr(node, "source", "") or cand.source
        template = [(k, v) for k, v in cand.template_params if k in source]
        kernel = cuda_kernel(
            name=getattr(node, "name", None) or "search_kernel",
            input_names=list(node.input_names),
            output_names=list(node.output_names),
            source=source,
            header=getattr(node, "header", "") or "",
        )
        out_shapes = [tuple(s) for s in node.output_shapes]
        out_dtypes = [dt.from_any(getattr(d, "value", d)) for d in node.output_dtypes]
        tg = cand.threadgroup

        def fn(*inputs):
            grid = self._grid(node, cand, inputs)
            cand.grid = grid
            outs = kernel(inputs=list(inputs), output_shapes=out_shapes, output_dtypes=out_dtypes,
                          grid=grid, threadgroup=tg if len(tg) == 3 else (tg[0], 1, 1),
                          template=template)
            return outs[0] if len(outs) == 1 else outs

        return fn
