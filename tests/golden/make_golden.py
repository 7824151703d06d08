"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a checkout that has the phew reference importable (default
/root/reference, or $PHEW_REFERENCE):

    python tests/golden/make_golden.py

Writes
* verdicts.json -- verdicts and failure strings of the reference's own
  ``EquivalenceChecker.check`` (verify/checker.py:77-218) on the cases of
  ``verdict_cases.py``; MLX is absent, so ``mlx.core`` is served by the
  oracle namespace (numpy) while the checker's code runs unchanged;
* allclose.json -- the reference's ``_allclose`` (checker.py:220-233) on
  seeded array pairs covering NaN/Inf/fp16/fp32 arithmetic;
* bench.json -- the reference's ``compare`` / ``check_convergence`` outputs;
* chains.json -- fused chains that the reference's ElementwiseFusionPass
  (rules/fusion.py:116-332) forms on the benchmark graphs;
* sources/*.py -- ``output_source`` of the reference's passes + MLXCodegen,
  re-targeted by ``phew_b200.integration`` (the drop-in binding).
"""

from __future__ import annotations

import json
import math
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = Path(os.environ.get("PHEW_REFERENCE", "/root/reference"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE))

from oracle import mlx_cpu  # noqa: E402


def fake_mlx():
    pkg = types.ModuleType("mlx")
    pkg.__path__ = []
    pkg.core = mlx_cpu
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = mlx_cpu


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
    # JSON cannot hold NaN/Inf portably: encode as strings
    for c in cases:
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
    for cur, cand, sizes, beaten in ((10, 9, 1, 1), (10, 9.9, 1, 1), (10, 5, 3, 1), (10, 5, 3, 3), (0, 1, 1, 1)):
        conv.append({"args": [cur, cand, sizes, beaten], "result": check_convergence(cur, cand, sizes, beaten)})
    return {"compare": rows, "convergence": conv}


# -- benchmark graphs built with the reference's IR (what its tracer records) --


def _graphs():
    from phew.ir import Constant, Dtype, Elementwise, Graph, Input, MatMul, Reduce, Transpose

    def ew(g, op, *ins, shape, dt):
        return g.add(Elementwise(shape=shape, dtype=dt, inputs=[i.id for i in ins], op=op))

    def const(g, v, dt):
        return g.add(Constant(shape=(), dtype=dt, value=v))

    def rms(n=1024):
        g = Graph()
        dt = Dtype.float32
        S = (n, 2048)
        x = g.add(Input(shape=S, dtype=dt, name="x"))
        w = g.add(Input(shape=(2048,), dtype=dt, name="w"))
        sq = ew(g, "mul", x, x, shape=S, dt=dt)
        m = g.add(Reduce(shape=(n, 1), dtype=dt, inputs=[sq.id], op="mean", axes=(1,), keepdims=True))
        a = ew(g, "add", m, const(g, 1e-5, dt), shape=(n, 1), dt=dt)
        r = ew(g, "rsqrt", a, shape=(n, 1), dt=dt)
        y = ew(g, "mul", x, r, shape=S, dt=dt)
        z = ew(g, "mul", y, w, shape=S, dt=dt)
        g.outputs = [z.id]
        return g

    def gelu(rows=4096):
        g = Graph()
        dt = Dtype.float16
        S = (rows, 8192)
        x = g.add(Input(shape=S, dtype=dt, name="x"))
        a = g.add(Input(shape=(8192,), dtype=dt, name="a"))
        b = g.add(Input(shape=(8192,), dtype=dt, name="b"))
        c = g.add(Input(shape=S, dtype=dt, name="c"))
        xa = ew(g, "mul", x, a, shape=S, dt=dt)
        y = ew(g, "add", xa, b, shape=S, dt=dt)
        yh = ew(g, "mul", y, const(g, 0.5, dt), shape=S, dt=dt)
        yy = ew(g, "mul", y, y, shape=S, dt=dt)
        yyy = ew(g, "mul", yy, y, shape=S, dt=dt)
        cub = ew(g, "mul", yyy, const(g, 0.044715, dt), shape=S, dt=dt)
        inner = ew(g, "add", y, cub, shape=S, dt=dt)
        arg = ew(g, "mul", inner, const(g, math.sqrt(2 / math.pi), dt), shape=S, dt=dt)
        t = ew(g, "tanh", arg, shape=S, dt=dt)
        t1 = ew(g, "add", t, const(g, 1.0, dt), shape=S, dt=dt)
        ge = ew(g, "mul", yh, t1, shape=S, dt=dt)
        s = ew(g, "sigmoid", c, shape=S, dt=dt)
        gs = ew(g, "mul", ge, s, shape=S, dt=dt)
        z = ew(g, "add", gs, x, shape=S, dt=dt)
        g.outputs = [z.id]
        return g

    def attn(L=2048):
        g = Graph()
        dt = Dtype.bfloat16
        S = (4, 32, L, 128)
        P = (4, 32, L, L)
        q = g.add(Input(shape=S, dtype=dt, name="q"))
        k = g.add(Input(shape=S, dtype=dt, name="k"))
        v = g.add(Input(shape=S, dtype=dt, name="v"))
        mask = g.add(Input(shape=(L, L), dtype=dt, name="mask"))
        kt = g.add(Transpose(shape=(4, 32, 128, L), dtype=dt, inputs=[k.id], axes=(0, 1, 3, 2)))
        s = g.add(MatMul(shape=P, dtype=dt, inputs=[q.id, kt.id]))
        sc = ew(g, "mul", s, const(g, 1 / math.sqrt(128), dt), shape=P, dt=dt)
        sm_in = ew(g, "add", sc, mask, shape=P, dt=dt)
        sm = g.add(Reduce(shape=P, dtype=dt, inputs=[sm_in.id], op="softmax", axes=(3,), keepdims=True))
        o = g.add(MatMul(shape=S, dtype=dt, inputs=[sm.id, v.id]))
        g.outputs = [o.id]
        return g

    def normed_mm(M=8192):
        g = Graph()
        dt = Dtype.bfloat16
        S = (M, 4096)
        x = g.add(Input(shape=S, dtype=dt, name="x"))
        W = g.add(Input(shape=(4096, 4096), dtype=dt, name="W"))
        mm = g.add(MatMul(shape=S, dtype=dt, inputs=[x.id, W.id]))
        sq = ew(g, "mul", x, x, shape=S, dt=dt)
        m = g.add(Reduce(shape=(M, 1), dtype=dt, inputs=[sq.id], op="mean", axes=(1,), keepdims=True))
        r = ew(g, "rsqrt", ew(g, "add", m, const(g, 1e-5, dt), shape=(M, 1), dt=dt), shape=(M, 1), dt=dt)
        z = ew(g, "mul", mm, r, shape=S, dt=dt)
        g.outputs = [z.id]
        return g

    return {"rms_norm": rms, "gelu_chain": gelu, "attention": attn, "normed_matmul": normed_mm}


def make_chains():
    from phew.rules.fusion import ElementwiseFusionPass

    from phew_b200.graph import from_phew

    out = {}
    for name, build in _graphs().items():
        g = build()
        spec = from_phew(g)
        p = ElementwiseFusionPass()
        chains = p._find_chains(g)
        recs = []
        for ch in chains:
            ids = {n.id for n in ch}
            ext_in, seen = [], set()
            from phew.ir.ops import Constant

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


def make_sources():
    from phew.rules import run_all_passes
    from phew.verify import SubstitutionClass as SC

    from phew_b200 import integration

    integration.install(mx_module=False)
    import phew.emit

    srcs = {}
    for name, build in _graphs().items():
        classes = {SC.fp32_to_fp32}
        if name == "normed_matmul":
            classes.add(SC.normed_matmul)
        for fusion in (False, True):
            g = build()
            g, applied = run_all_passes(g, enable_tensorops=False, enable_fusion=fusion,
                                        enabled_subst_classes=classes)
            src = phew.emit.MLXCodegen().emit(g, fn_name="optimized")
            key = f"{name}__fusion{int(fusion)}"
            srcs[key] = {"applied": applied, "source": src}
    return srcs


def main() -> int:
    fake_mlx()
    (HERE / "sources").mkdir(exist_ok=True)
    (HERE / "verdicts.json").write_text(json.dumps(make_verdicts(), indent=1))
    (HERE / "allclose.json").write_text(json.dumps(make_allclose()))
    (HERE / "bench.json").write_text(json.dumps(make_bench(), indent=1))
    (HERE / "chains.json").write_text(json.dumps(make_chains()))
    srcs = make_sources()
    index = {}
    for key, rec in srcs.items():
        (HERE / "sources" / f"{key}.py").write_text(rec["source"])
        index[key] = rec["applied"]
    (HERE / "sources" / "index.json").write_text(json.dumps(index, indent=1))
    print("wrote fixtures to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
