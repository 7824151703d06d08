"""End to end on the GPU: phew's emitted ``output_source`` (golden fixtures
produced by the reference's passes and MLXCodegen, re-targeted to this
backend) and the unoptimised harness functions, against the oracle."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import mlx_cpu
from phew_b200.workloads import WORKLOADS

pytestmark = pytest.mark.gpu

SOURCES = Path(__file__).resolve().parent / "golden" / "sources"
RTOL = {"float32": 1e-5, "float16": 2e-2, "bfloat16": 2e-2}
ATOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 2e-2}


def load_source(key: str):
    ns: dict = {}
    exec(compile((SOURCES / f"{key}.py").read_text(), f"<{key}>", "exec"), ns)
    return ns["optimized"]


def run_and_compare(mx, name, fn, size, seed=0):
    w = WORKLOADS[name]
    host = w.host_inputs(size, seed)
    got = fn(*[mx.array(a) for a in host])
    ref = w.make_fn(mlx_cpu)(*[mlx_cpu.array(a) for a in host])
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    assert g.shape == r.shape
    np.testing.assert_allclose(g, r, rtol=RTOL[w.dtype], atol=ATOL[w.dtype])
    return g, r


@pytest.mark.parametrize("key", ["rms_norm__fusion0", "rms_norm__fusion1"])
@pytest.mark.parametrize("size", ["small", "typical", "large"])
def test_rms_norm_candidates(mx, key, size):
    run_and_compare(mx, "rms_norm", load_source(key), size)


@pytest.mark.parametrize("key", ["gelu_chain__fusion0", "gelu_chain__fusion1"])
@pytest.mark.parametrize("size", ["small", "typical"])
def test_gelu_chain_candidates(mx, key, size):
    g, r = run_and_compare(mx, "gelu_chain", load_source(key), size, seed=1)
    assert np.mean(g == r) > 0.97  # per-node rounding reproduced


@pytest.mark.parametrize("name", ["rms_norm", "gelu_chain"])
def test_baseline_functions(mx, name):
    w = WORKLOADS[name]
    run_and_compare(mx, name, w.make_fn(mx), "small", seed=2)


def test_verify_fused_candidate_passes(mx):
    """The reference's verification protocol accepts the fused rms_norm
    candidate against its unfused baseline on this backend."""
    from phew_b200.verify import EquivalenceChecker

    w = WORKLOADS["rms_norm"]
    res = EquivalenceChecker(n_seeds=2).check(w.make_fn(mx), load_source("rms_norm__fusion1"),
                                              w.input_factory(mx))
    assert res.passed, res.failures
