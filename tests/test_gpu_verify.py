"""GPU verdicts: the device comparison and the equivalence checker reproduce
the reference's verdicts (golden fixtures made by running the reference's
own checker code)."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import mlx_cpu, verdict

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import verdict_cases  # noqa: E402


def _vals(xs):
    return np.array([float(x) if isinstance(x, str) else x for x in xs], dtype=np.float64)


def test_compare_allclose_golden(mx):
    from phew_b200.verify import compare_arrays

    for c in json.loads((GOLDEN / "allclose.json").read_text()):
        a = _vals(c["a"]).astype(c["dtype"])
        b = _vals(c["b"]).astype(c["dtype"])
        st = compare_arrays(mx.array(a), mx.array(b), c["atol"], c["rtol"])
        # the golden rule has no skip: a non-finite baseline is skipped by the
        # checker before _allclose runs
        if not np.all(np.isfinite(a)):
            assert st.skipped == 1
            continue
        assert bool(st.passed) == c["ok"], (c["dtype"], c["kind"], c["atol"])


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("scale", [1.0, 1e-6, 1e6, 2e10])
@pytest.mark.parametrize("perturb", [0.0, 1e-5, 3e-3, 0.1])
def test_compare_matches_restated_rule(mx, dtype, scale, perturb):
    from phew_b200.verify import compare_arrays

    rng = np.random.default_rng(int(scale) % 1000 + int(perturb * 1e5))
    npd = mlx_cpu._NP[dtype]
    b = (rng.standard_normal(5000).astype(np.float32) * scale).astype(npd)
    c = (b.astype(np.float64) * (1 + perturb * rng.standard_normal(5000))).astype(np.float32).astype(npd)
    tol = verdict.TOLERANCES["fp32_to_fp32"]
    is_bf16 = dtype == "bfloat16"
    b_np = b.astype(np.float32) if is_bf16 else b
    c_np = c.astype(np.float32) if is_bf16 else c
    want = verdict.compare_output(b_np, c_np, tol, is_bf16)
    st = compare_arrays(mx.array(b), mx.array(c), tol.atol, tol.rtol)
    assert bool(st.passed) == want.ok
    assert bool(st.skipped) == want.skipped
    if not want.ok:
        assert st.max_abs_diff == pytest.approx(want.max_diff, rel=1e-12)
        assert st.n_mismatch > 0


def test_compare_nan_positions(mx):
    from phew_b200.verify import compare_arrays

    b = np.arange(100, dtype=np.float32)
    c = b.copy()
    c[10] = np.nan
    st = compare_arrays(mx.array(b), mx.array(c), 1e-5, 1e-5)
    assert not st.passed and st.n_nan_any == 1 and st.n_mismatch == 1
    b2 = b.copy()
    b2[3] = np.inf
    st = compare_arrays(mx.array(b2), mx.array(c), 1e-5, 1e-5)
    assert st.skipped and st.passed


def test_compare_is_deterministic_across_sizes(mx):
    from phew_b200.verify import compare_arrays

    rng = np.random.default_rng(3)
    b = rng.standard_normal(3_000_001).astype(np.float32)
    s1 = compare_arrays(mx.array(b), mx.array(b), 1e-5, 1e-5)
    s2 = compare_arrays(mx.array(b), mx.array(b), 1e-5, 1e-5)
    assert s1.sum_abs_base == s2.sum_abs_base  # bitwise identical
    assert s1.sum_abs_base == pytest.approx(float(np.abs(b.astype(np.float64)).sum()), rel=1e-12)


@pytest.mark.parametrize("case", verdict_cases.CASES, ids=[c[0] for c in verdict_cases.CASES])
def test_checker_verdicts_match_reference(mx, case):
    from phew_b200.verify import EquivalenceChecker, SubstitutionClass

    golden = {g["name"]: g for g in json.loads((GOLDEN / "verdicts.json").read_text())}
    name, classes, base, cand, factory = verdict_cases.build(case, mx)
    res = EquivalenceChecker(enabled_classes={SubstitutionClass(c) for c in classes}).check(
        base, cand, factory)
    assert res.passed == golden[name]["passed"]
    assert res.failures == golden[name]["failures"]


def test_checker_rejects_disabled_class(mx):
    from phew_b200.verify import EquivalenceChecker, SubstitutionClass

    chk = EquivalenceChecker(subst_class=SubstitutionClass.fp32_to_fp16,
                             enabled_classes={SubstitutionClass.fp32_to_fp32})
    res = chk.check(lambda: None, lambda: None, lambda s, k: ([], {}))
    assert not res.passed and "opt-in" in res.failures[0].lower()
