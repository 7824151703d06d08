"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run with the phew reference checkout named by $PHEW_REFERENCE (or with its
``phew`` package importable):

    python tests/golden/make_golden.py

The reference's numerics need MLX, which is not installable here; its
Python code (tracer, passes, emitter, checker) runs unchanged with
``mlx.core`` served by the oracle namespace (``oracle/mlx_cpu.py``).

Writes
* verdicts.json -- verdicts and failure strings of the reference's own
  ``EquivalenceChecker.check`` (verify/checker.py:77-218) on the cases of
  ``verdict_cases.py``;
* allclose.json -- the reference's ``_allclose`` (checker.py:220-233) on
  seeded array pairs covering NaN/Inf/fp16/fp32 arithmetic;
* bench.json -- the reference's ``compare`` / ``check_convergence`` outputs;
* chains.json -- fused chains that the reference's ElementwiseFusionPass
  (rules/fusion.py:116-332) forms on the benchmark graphs;
* sources/*.py -- ``output_source`` of the reference's tracer + passes +
  MLXCodegen, re-targeted by ``phew_b200.integration`` (the drop-in
  binding), for the benchmark functions and for the 16 decoder-block
  candidates of the verification sweep (rms_norm / SDPA / normed-matmul
  substitution x elementwise fusion, on or off);
* sources/cuda_chains.json -- for every fused kernel body in those sources,
  the chain it was emitted from, so the oracle can evaluate it on the CPU;
* op_registry.json -- the mlx.core / mlx.core.fast op names the reference's
  tracer records (ir/op_registry.py), which the backend's mx namespace must
  provide;
* optimizer_runs.json -- the reference's own ``Optimizer(fn,
  input_factory).run()`` (optimizer.py:90-353) on the rms_norm and
  gelu_chain harnesses with elementwise fusion off (the fused kernels' MSL
  cannot run on the oracle): the rules it applied, its Step-7 verdict, its
  ``output_source`` and the step names of its search trace.

``python tests/golden/make_golden.py --part optimizer`` regenerates only
that file.
"""

from __future__ import annotations

import hashlib
import itertools
import json
import math
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
def _reference_root() -> Path:
    env = os.environ.get("PHEW_REFERENCE")
    if env:
        return Path(env)
    import importlib.util

    spec = importlib.util.find_spec("phew")
    if spec is None or not spec.origin:
        raise SystemExit("make_golden: set PHEW_REFERENCE to the phew reference checkout")
    return Path(spec.origin).resolve().parent.parent


REF = _reference_root()
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE))

from oracle import mlx_cpu  # noqa: E402

from phew_b200 import workloads as W  # noqa: E402

SOURCES = HERE / "sources"


def fake_mlx():
    """Register an ``mlx`` package whose ``core`` is the oracle namespace."""
    core = types.ModuleType("mlx.core")
    for k in dir(mlx_cpu):
        if not k.startswith("__"):
            setattr(core, k, getattr(mlx_cpu, k))
    # dtype names the reference's Dtype.from_mlx table expects (ir/dtype.py:70-88)
    core.float64 = mlx_cpu.Dtype("float32")
    core.complex64 = mlx_cpu.Dtype("float32")
    fast = types.ModuleType("mlx.core.fast")
    fast.rms_norm = mlx_cpu.rms_norm
    fast.scaled_dot_product_attention = mlx_cpu.fast.scaled_dot_product_attention
    core.fast = fast
    nn = types.ModuleType("mlx.nn")
    pkg = types.ModuleType("mlx")
    pkg.__path__ = []
    pkg.core, pkg.nn = core, nn
    sys.modules.update({"mlx": pkg, "mlx.core": core, "mlx.core.fast": fast, "mlx.nn": nn})
    return core


def placeholder(shape, dtype):
    """A zero-cost oracle array of the given shape (the tracer reads only
    shapes and dtypes)."""
    d = mlx_cpu.as_dtype(dtype)
    return mlx_cpu.array.wrap(np.broadcast_to(np.zeros((), d.np), shape), d)


def trace(fn, shapes_dtypes):
    from phew.ir.importer import trace_to_graph

    return trace_to_graph(fn, [placeholder(s, d) for s, d in shapes_dtypes], {})


# ---------------------------------------------------------------------------
# verdict / bench goldens
# ---------------------------------------------------------------------------


def make_verdicts():
    import verdict_cases
    from phew.verify import EquivalenceChecker, SubstitutionClass

    out = []
    for case in verdict_cases.CASES:
        name, classes, base, cand, factory = verdict_cases.build(case, mlx_cpu)
        enabled = {SubstitutionClass(c) for c in classes}
        res = EquivalenceChecker(enabled_classes=enabled).check(base, cand, factory)
        out.append({"name": name, "classes": classes, "passed": res.passed,
                    "failures": res.failures, "atol": res.tolerance.atol,
                    "rtol": res.tolerance.rtol})
    return out


def make_allclose():
    from phew.verify import EquivalenceChecker
    from phew.verify.tolerances import Tolerance

    chk = EquivalenceChecker()
    rng = np.random.default_rng(7)
    cases = []
    for dtype in ("float32", "float16"):
        for kind in ("near", "far", "nan_same", "nan_diff", "inf", "tiny"):
            a = rng.standard_normal(64).astype(dtype)
            b = a.copy()
            if kind == "near":
                b = (a.astype(np.float64) * (1 + 4e-6)).astype(dtype)
            elif kind == "far":
                b = (a.astype(np.float64) * 1.01).astype(dtype)
            elif kind == "nan_same":
                a[3] = np.nan
                b[3] = np.nan
            elif kind == "nan_diff":
                b[5] = np.nan
            elif kind == "inf":
                b[7] = np.inf
            elif kind == "tiny":
                a = (a * 1e-6).astype(dtype)
                b = (a.astype(np.float64) + 9e-6).astype(dtype)
            for atol, rtol in ((1e-5, 1e-5), (1e-3, 1e-2), (1e-2, 5e-2)):
                ok = chk._allclose(a, b, tol=Tolerance(atol=atol, rtol=rtol, opt_in=False))
                cases.append({"dtype": dtype, "kind": kind, "atol": atol, "rtol": rtol,
                              "a": a.astype(np.float64).tolist(), "b": b.astype(np.float64).tolist(),
                              "ok": bool(ok)})
    for c in cases:  # JSON cannot hold NaN/Inf portably: encode as strings
        for k in ("a", "b"):
            c[k] = [repr(v) if not math.isfinite(v) else v for v in c[k]]
    return cases


def make_bench():
    from phew.bench.convergence import check_convergence
    from phew.bench.harness import BenchResult, compare

    rows = []
    for bm, om in ((10.0, 5.0), (10.0, 9.9), (10.0, 10.31), (1.0, 0.9)):
        b = BenchResult(bm, 0.1, 0.01, 20, True, [bm])
        o = BenchResult(om, 0.1, 0.01, 20, False, [om])
        rows.append({"baseline": bm, "optimized": om, "compare": compare(b, o)})
    conv = []
    for args in ((10, 9, 1, 1), (10, 9.9, 1, 1), (10, 5, 3, 1), (10, 5, 3, 3), (0, 1, 1, 1)):
        conv.append({"args": list(args), "result": check_convergence(*args)})
    return {"compare": rows, "convergence": conv}


# ---------------------------------------------------------------------------
# graphs of the benchmark functions, traced by the reference's tracer
# ---------------------------------------------------------------------------


def graphs(core):
    bf, f16, f32 = "bfloat16", "float16", "float32"
    dec_full = W.decoder_arg_shapes(W.DECODER_SEQ["typical"], W.DECODER_FULL)
    dec_tiny = W.decoder_arg_shapes(W.DECODER_TINY_SEQ["typical"], W.DECODER_TINY)
    return {
        "rms_norm": lambda: trace(W.rms_norm_fn(core), [((1024, 2048), f32), ((2048,), f32)]),
        "gelu_chain": lambda: trace(W.gelu_chain_fn(core), [((4096, 8192), f16), ((8192,), f16),
                                                             ((8192,), f16), ((4096, 8192), f16)]),
        "attention": lambda: trace(W.attention_fn(core), [((4, 32, 2048, 128), bf)] * 3 +
                                   [((2048, 2048), bf)]),
        "normed_matmul": lambda: trace(W.normed_matmul_fn(core), [((8192, 4096), bf),
                                                                  ((4096, 4096), bf)]),
        "layer_norm": lambda: trace(W.layer_norm_fn(core), [((1024, 2048), f32), ((2048,), f32),
                                                             ((2048,), f32)]),
        "rope": lambda: trace(W.rope_fn(core), [((8, 32, 2048, 128), bf), ((2048, 64), bf)]),
        "decoder_full": lambda: trace(W.decoder_block_fn(core, W.DECODER_FULL), [(s, bf) for s in dec_full]),
        "decoder_tiny": lambda: trace(W.decoder_block_fn(core, W.DECODER_TINY), [(s, bf) for s in dec_tiny]),
    }


def make_chains(core):
    from phew.ir.ops import Constant
    from phew.rules.fusion import ElementwiseFusionPass

    from phew_b200.graph import from_phew

    out = {}
    for name, build in graphs(core).items():
        if name.startswith("decoder"):
            continue
        g = build()
        spec = from_phew(g)
        recs = []
        for ch in ElementwiseFusionPass()._find_chains(g):
            ids = {n.id for n in ch}
            ext_in, seen = [], set()
            for n in ch:
                if isinstance(n, Constant):
                    continue
                for i in n.inputs:
                    if i not in ids and i not in seen and i in g:
                        ext_in.append(i)
                        seen.add(i)
            outs = [n.id for n in ch if not isinstance(n, Constant) and (
                n.id in g.outputs or any(s.id not in ids for s in g.successors(n.id)))]
            recs.append({"nodes": [n.id for n in ch], "ext_inputs": ext_in, "ext_outputs": outs})
        out[name] = {"graph": spec.to_json(), "chains": recs}
    return out


# ---------------------------------------------------------------------------
# candidates
# ---------------------------------------------------------------------------


def apply_candidate(graph, rms: bool, sdpa: bool, nmm: bool, fusion: bool):
    """The reference's pass order (rules/graph_passes.py:24-114) with each
    primitive substitution toggled on its own.  With every toggle on this is
    run_all_passes(enable_fusion=fusion, normed_matmul enabled)."""
    from phew.rules.algebraic import AlgebraicPass
    from phew.rules.compile_boundaries import CompileBoundaryPass
    from phew.rules.fusion import ElementwiseFusionPass
    from phew.rules.primitive_subst import PrimitiveSubstPass
    from phew.verify import SubstitutionClass as SC

    applied = []
    before = len(graph)
    AlgebraicPass().run(graph)
    if len(graph) != before:
        applied.append("algebraic")
    if fusion and ElementwiseFusionPass().run(graph):
        applied.append("elementwise_fusion")
    if CompileBoundaryPass().run(graph):
        applied.append("compile_boundary")
    p = PrimitiveSubstPass(enabled_classes={SC.fp32_to_fp32, SC.normed_matmul})
    changed = False
    if rms:
        changed |= p._match_rms_norm(graph)
    if nmm:
        changed |= p._match_normed_matmul(graph)
    changed |= p._match_layer_norm(graph)
    changed |= p._match_rope(graph)
    if sdpa:
        changed |= p._match_sdpa(graph)
    if changed:
        applied.append("primitive_subst")
    return graph, applied


class ChainRecorder:
    """Wraps the CUDA emitter to remember the chain behind every body."""

    def __init__(self):
        from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen
        from phew_b200.graph import from_phew  # noqa: F401

        self.base = SubgraphCUDACodegen
        self.chains = {}
        rec = self

        class Recording(SubgraphCUDACodegen):
            def emit(self, nodes, ext_in, ext_out):
                src, i, o = super().emit(nodes, ext_in, ext_out)
                rec.chains[hashlib.sha1(src.encode()).hexdigest()] = {
                    "nodes": [_node_json(n) for n in nodes],
                    "ext_inputs": [_node_json(n) for n in ext_in],
                    "ext_outputs": [_node_json(n) for n in ext_out],
                }
                return src, i, o

        self.cls = Recording


def _node_json(n):
    from phew_b200.graph import from_phew

    class One:
        def __init__(self, node):
            self._n = [node]
            self.outputs = [node.id]

        def nodes(self):
            return self._n

    return from_phew(One(n)).to_json()["nodes"][0]


def make_sources(core):
    from phew.rules import run_all_passes
    from phew.verify import SubstitutionClass as SC

    from phew_b200 import integration

    integration.install(mx_module=False)
    import phew.emit
    import phew.emit.msl_codegen

    rec = ChainRecorder()
    phew.emit.msl_codegen.SubgraphMSLCodegen = rec.cls
    builders = graphs(core)
    srcs = {}
    for name in ("rms_norm", "gelu_chain", "attention", "normed_matmul", "layer_norm", "rope"):
        classes = {SC.fp32_to_fp32}
        if name == "normed_matmul":
            classes.add(SC.normed_matmul)
        for fusion in (False, True):
            g, applied = run_all_passes(builders[name](), enable_tensorops=False,
                                        enable_fusion=fusion, enabled_subst_classes=classes)
            srcs[f"{name}__fusion{int(fusion)}"] = (applied, phew.emit.MLXCodegen().emit(g, fn_name="optimized"))
    for name in ("decoder_full", "decoder_tiny"):
        for rms, sdpa, nmm, fusion in itertools.product((0, 1), repeat=4):
            g, applied = apply_candidate(builders[name](), bool(rms), bool(sdpa), bool(nmm), bool(fusion))
            key = f"{name}__rms{rms}_sdpa{sdpa}_nmm{nmm}_fus{fusion}"
            srcs[key] = (applied, phew.emit.MLXCodegen().emit(g, fn_name="optimized"))
    phew.emit.msl_codegen.SubgraphMSLCodegen = rec.base
    return srcs, rec.chains


def make_op_registry():
    """The reference tracer's op coverage (ir/op_registry.py): the mlx.core
    and mlx.core.fast names it records, which this backend must provide."""
    from phew.ir import op_registry as R

    return {"IMPLEMENTED": sorted(R.IMPLEMENTED), "FAST_IMPLEMENTED": sorted(R.FAST_IMPLEMENTED)}


# Rows per size of the Optimizer runs: the oracle evaluates every op on the
# CPU, and the reference's benchmark calls each function up to ~850 times in
# one run, so the runs use fewer rows than the benchmark shapes (the emitted
# sources do not depend on the row count).
OPTIMIZER_ROWS = {"rms_norm": {"small": 8, "typical": 32, "large": 128},
                  "gelu_chain": {"small": 4, "typical": 16, "large": 64}}


def optimizer_inputs(name, size, seed):
    rows = OPTIMIZER_ROWS[name][size]
    if name == "rms_norm":
        return W.rms_norm_inputs(size, seed, rows=rows)
    return W.gelu_chain_inputs(size, seed, rows=rows)


def make_optimizer_runs(core):
    """Run the reference's Optimizer end to end with mlx.core served by the
    oracle (the reference's own benchmark, passes, codegen and checker; no
    part of this backend is installed)."""
    import time

    from phew.optimizer import Optimizer

    if not hasattr(core, "metal"):
        core.metal = types.SimpleNamespace(is_available=lambda: False)
    runs = {}
    for name in ("rms_norm", "gelu_chain"):
        w = W.WORKLOADS[name]

        def factory(size, seed, name=name):
            return [core.array(a) for a in optimizer_inputs(name, size, seed)], {}

        t0 = time.perf_counter()
        res = Optimizer(w.make_fn(core), factory, enable_elementwise_fusion=False).run()
        print(f"optimizer run {name}: {time.perf_counter() - t0:.1f} s", flush=True)
        runs[f"{name}__fusion0"] = {
            "rows": OPTIMIZER_ROWS[name],
            "applied_rules": list(res.applied_rules),
            "verification_passed": bool(res.verification_passed),
            "verification_details": list(res.verification_details),
            "output_source": res.output_source,
            "steps": [ln for ln in res.search_trace if ln.startswith("Step")],
        }
    return runs


def main() -> int:
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--part", choices=["all", "optimizer"], default="all")
    args = ap.parse_args()
    core = fake_mlx()
    # before make_sources, which re-targets phew's codegen to this backend
    (HERE / "optimizer_runs.json").write_text(json.dumps(make_optimizer_runs(core), indent=1))
    if args.part == "optimizer":
        print(f"wrote {HERE / 'optimizer_runs.json'}")
        return 0
    (HERE / "op_registry.json").write_text(json.dumps(make_op_registry(), indent=1))
    SOURCES.mkdir(exist_ok=True)
    (HERE / "verdicts.json").write_text(json.dumps(make_verdicts(), indent=1))
    (HERE / "allclose.json").write_text(json.dumps(make_allclose()))
    (HERE / "bench.json").write_text(json.dumps(make_bench(), indent=1))
    (HERE / "chains.json").write_text(json.dumps(make_chains(core)))
    srcs, chains = make_sources(core)
    index = {}
    for key, (applied, src) in srcs.items():
        (SOURCES / f"{key}.py").write_text(src)
        index[key] = applied
    (SOURCES / "index.json").write_text(json.dumps(index, indent=1))
    (SOURCES / "cuda_chains.json").write_text(json.dumps(chains))
    print(f"wrote {len(srcs)} sources and {len(chains)} fused chains to {HERE}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
