"""The oracle against the reference's own golden outputs, and its internal
consistency (CPU only)."""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import mlx_cpu, verdict

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import verdict_cases  # noqa: E402


def _vals(xs):
    return np.array([float(x) if isinstance(x, str) else x for x in xs], dtype=np.float64)


def test_allclose_matches_reference():
    cases = json.loads((GOLDEN / "allclose.json").read_text())
    assert len(cases) >= 30
    for c in cases:
        a = _vals(c["a"]).astype(c["dtype"])
        b = _vals(c["b"]).astype(c["dtype"])
        assert verdict.allclose(a, b, c["atol"], c["rtol"]) == c["ok"], c["kind"]


@pytest.mark.parametrize("case", verdict_cases.CASES, ids=[c[0] for c in verdict_cases.CASES])
def test_check_loop_matches_reference(case):
    golden = {g["name"]: g for g in json.loads((GOLDEN / "verdicts.json").read_text())}
    name, classes, base, cand, factory = verdict_cases.build(case, mlx_cpu)
    passed, failures = verdict.check(base, cand, factory, mlx_cpu, set(classes))
    assert passed == golden[name]["passed"]
    assert failures == golden[name]["failures"]


def test_tolerance_table_matches_product():
    from phew_b200.verify import TOLERANCES, SubstitutionClass

    for k, t in verdict.TOLERANCES.items():
        p = TOLERANCES[SubstitutionClass(k)]
        assert (p.atol, p.rtol, p.opt_in) == (t.atol, t.rtol, t.opt_in)


def test_bench_logic_matches_reference():
    from phew_b200.bench import BenchResult, check_convergence, compare

    g = json.loads((GOLDEN / "bench.json").read_text())
    for row in g["compare"]:
        b = BenchResult(row["baseline"], 0.1, 0.01, 20, True, [row["baseline"]])
        o = BenchResult(row["optimized"], 0.1, 0.01, 20, False, [row["optimized"]])
        got = compare(b, o)
        for k, v in row["compare"].items():
            assert math.isclose(got[k], v, rel_tol=1e-12), k
    for row in g["convergence"]:
        assert check_convergence(*row["args"]) == row["result"]


def test_eval_chain_equals_op_by_op():
    from phew_b200.workloads import gelu_chain_fn, gelu_chain_inputs, gelu_chain_nodes

    xs = gelu_chain_inputs("small", 3, rows=16)
    chain, ins, outs = gelu_chain_nodes(16)
    fused = mlx_cpu.eval_chain(chain, ins, outs, xs)[0]
    fn = gelu_chain_fn(mlx_cpu)
    ref = np.asarray(fn(*[mlx_cpu.array(a) for a in xs]))
    assert fused.dtype == np.float16
    np.testing.assert_array_equal(fused, ref)


def test_weak_scalars_take_array_dtype():
    x = mlx_cpu.array(np.array([1.0, 2.0], np.float16))
    y = x * 0.1
    assert y.dtype is mlx_cpu.float16
    assert np.asarray(y)[0] == np.float16(np.float16(0.1) * np.float16(1.0))


def test_rms_norm_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 64)).astype(np.float32)
    w = rng.standard_normal(64).astype(np.float32)
    y = np.asarray(mlx_cpu.rms_norm(mlx_cpu.array(x), mlx_cpu.array(w), 1e-5))
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, -1, keepdims=True) + 1e-5) * w
    np.testing.assert_allclose(y, ref, rtol=2e-6, atol=1e-6)


def test_sdpa_causal_masks_future():
    rng = np.random.default_rng(1)
    q = mlx_cpu.array(rng.standard_normal((1, 1, 4, 8)).astype(np.float32))
    k = mlx_cpu.array(rng.standard_normal((1, 1, 4, 8)).astype(np.float32))
    v = mlx_cpu.array(rng.standard_normal((1, 1, 4, 8)).astype(np.float32))
    o = np.asarray(mlx_cpu.sdpa(q, k, v, 0.35, "causal"))
    # first query attends only to the first key
    np.testing.assert_allclose(o[0, 0, 0], np.asarray(v)[0, 0, 0], rtol=1e-6)
