"""Binding this backend into an unchanged phew installation.

``install()`` re-targets the four places where phew's candidate path reaches
the device, leaving the rest of phew (tracer, μGraph, passes, e-graph,
``Optimizer``) as it is:

1. fused-chain emission: ``ElementwiseFusionPass._fuse_chain`` imports
   ``SubgraphMSLCodegen`` from ``phew.emit.msl_codegen`` at call time
   (``rules/fusion.py:207,266-268``); it now gets :class:`SubgraphCUDACodegen`.
2. ``output_source``: ``MLXCodegen`` (``emit/codegen.py:26-57``) is kept as
   the producer; :class:`CUDAMLXCodegen` only swaps the ``mlx`` imports for
   ``phew_b200.mx`` and re-targets the kernel call sites of
   ``_emit_metal_kernel`` (``:478-600``) to ``mx.fast.cuda_kernel`` with this
   backend's grid policy.
3. ``benchmark`` / ``compare`` (``bench/harness.py:28-112``) -> CUDA-event
   timing in :mod:`phew_b200.bench`.
4. ``EquivalenceChecker`` (``verify/checker.py:46-263``) -> device-side
   comparison in :mod:`phew_b200.verify`.

``mlx.core`` itself is provided by ``phew_b200.mx`` (registered in
``sys.modules`` when no real MLX is importable), so ``Optimizer.run`` and
emitted code resolve ``mx`` to this backend.
"""

from __future__ import annotations

import re
import sys
import types

from .emit.cuda_codegen import SubgraphCUDACodegen

_GRID_RE = re.compile(r"^(\s*)grid=\((?P<expr>[^,]+\.size), 1, 1\),\s*$")


def cuda_codegen_class():
    """Subclass of phew's ``MLXCodegen`` whose output runs on this backend."""
    from phew.emit.codegen import MLXCodegen

    class CUDAMLXCodegen(MLXCodegen):
        def emit(self, graph, fn_name: str = "optimized") -> str:
            src = super().emit(graph, fn_name)
            src = src.replace("import mlx.core as mx\n", "import phew_b200.mx as mx\n", 1)
            src = src.replace("import mlx.core.fast as fast\n", "from phew_b200.mx import fast\n", 1)
            return src

        def _emit_metal_kernel(self, node, ins, vname, kernel_out_map):
            lines = super()._emit_metal_kernel(node, ins, vname, kernel_out_map)
            fused = bool(getattr(node, "attrs", {}).get("fusion_generated"))
            out = []
            for line in lines:
                line = line.replace("mx.fast.metal_kernel(", "mx.fast.cuda_kernel(")
                m = _GRID_RE.match(line)
                if fused and m:
                    line = f"{m.group(1)}grid=(mx.elementwise_threads({m.group('expr')}), 1, 1),"
                out.append(line)
            return out

    return CUDAMLXCodegen


def install_mx_module() -> None:
    """Make ``import mlx.core`` resolve to ``phew_b200.mx`` when MLX is absent."""
    try:
        import mlx.core  # noqa: F401

        return
    except ImportError:
        pass
    from . import mx as bmx

    pkg = types.ModuleType("mlx")
    pkg.__path__ = []  # a package
    pkg.core = bmx
    nn = types.ModuleType("mlx.nn")
    nn.silu = bmx.silu
    nn.gelu = bmx.gelu
    nn.relu = bmx.relu
    nn.softmax = bmx.softmax
    nn.sigmoid = bmx.sigmoid
    pkg.nn = nn
    sys.modules.setdefault("mlx", pkg)
    sys.modules.setdefault("mlx.core", bmx)
    sys.modules.setdefault("mlx.core.fast", bmx.fast)
    sys.modules.setdefault("mlx.nn", nn)


def install(mx_module: bool = True) -> None:
    """Re-target an importable phew to this backend (idempotent)."""
    import phew.bench
    import phew.emit
    import phew.emit.codegen
    import phew.emit.msl_codegen
    import phew.verify

    from . import bench as bbench
    from . import verify as bverify

    if mx_module:
        install_mx_module()
    phew.emit.msl_codegen.SubgraphMSLCodegen = SubgraphCUDACodegen
    cls = cuda_codegen_class()
    phew.emit.MLXCodegen = cls
    phew.emit.codegen.MLXCodegen = cls
    phew.bench.benchmark = bbench.benchmark
    phew.bench.compare = bbench.compare
    phew.verify.EquivalenceChecker = bverify.EquivalenceChecker
    # Phase-2 launch search (optimizer.py:250-279 imports it from phew.emit)
    from .emit.autotune import KernelParamSearch

    phew.emit.KernelParamSearch = KernelParamSearch
    try:
        import phew.emit.metal_kernel

        phew.emit.metal_kernel.KernelParamSearch = KernelParamSearch
    except ImportError:
        pass
