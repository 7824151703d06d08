"""ORACLE -- test infrastructure only (see oracle/mlx_cpu.py header).

Restatement of the reference equivalence checker's per-output rule and edge
variants, on numpy arrays, so the device comparison (``phew_compare``) and
the sweep's verdicts can be checked against it.  Pinned against the
reference's own functions by ``tests/golden/verdicts.json``.

Follows phew ``verify/checker.py``:
* ``compare_output``  <- the per-output loop body, :144-203
* ``allclose``        <- ``_allclose``, :220-233
* ``edge_variants``   <- ``_edge_variants``, :235-263
* ``TOLERANCES``      <- ``verify/tolerances.py:27-36``
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Tolerance:
    atol: float
    rtol: float
    opt_in: bool


TOLERANCES = {
    "fp32_to_fp32": Tolerance(1e-5, 1e-5, False),
    "fp32_to_fp16": Tolerance(1e-3, 1e-2, True),
    "fp32_to_bf16": Tolerance(1e-2, 1e-2, True),
    "quantized_4bit": Tolerance(1e-2, 5e-2, True),
    "normed_matmul": Tolerance(1e-3, 1e-1, True),
}


def checker_tolerance(enabled: set[str]) -> Tolerance:
    """The loosest enabled tolerance by atol (checker.py:71-75)."""
    cands = [TOLERANCES[c] for c in enabled if c in TOLERANCES]
    if not cands:
        return TOLERANCES["fp32_to_fp32"]
    return max(cands, key=lambda t: t.atol)


def allclose(a: np.ndarray, b: np.ndarray, atol: float, rtol: float) -> bool:
    nan_match = np.isnan(a) == np.isnan(b)
    finite_close = np.isclose(
        np.where(np.isnan(a), 0, a), np.where(np.isnan(b), 0, b), atol=atol, rtol=rtol
    )
    return bool(np.all(nan_match & (np.isnan(a) | finite_close)))


@dataclass
class OutputVerdict:
    ok: bool
    skipped: bool
    max_diff: float
    atol: float
    rtol: float


def compare_output(b_np: np.ndarray, c_np: np.ndarray, tol: Tolerance, is_bf16: bool) -> OutputVerdict:
    """One baseline/candidate output pair; `b_np`/`c_np` as the checker holds
    them (bf16 already widened to float32, float16 kept as float16)."""
    if not np.all(np.isfinite(b_np)):
        return OutputVerdict(True, True, 0.0, tol.atol, tol.rtol)
    atol, rtol = tol.atol, tol.rtol
    if is_bf16:
        out_mean = float(np.mean(np.abs(b_np)))
        if out_mean > 1e10:
            return OutputVerdict(True, True, 0.0, atol, rtol)
        f = 0.30 if out_mean > 1e6 else 0.05
        atol, rtol = max(atol, out_mean * f), max(rtol, f)
    if allclose(b_np, c_np, atol, rtol):
        return OutputVerdict(True, False, 0.0, atol, rtol)
    diff = float(np.max(np.abs(b_np.astype(np.float64) - c_np.astype(np.float64))))
    return OutputVerdict(False, False, diff, atol, rtol)


def edge_variants(args: list, seed: int, as_array=None):
    """Yield (name, args) like the reference: random, zeros, x1e-6, x1e6.

    `args` entries with a ``shape`` are arrays (numpy arrays or objects whose
    ``dtype`` converts with ``np.dtype``); `as_array(ndarray, like)` builds the
    variant array in the caller's array type (default: numpy cast to like's
    dtype).
    """
    def conv(v, like):
        if as_array is not None:
            return as_array(v, like)
        return np.asarray(v).astype(np.asarray(like).dtype)

    yield "random", list(args)
    yield "zeros", [conv(np.zeros(a.shape, np.float32), a) if hasattr(a, "shape") else a for a in args]
    rng = np.random.default_rng(seed + 1000)
    small = [conv(rng.standard_normal(a.shape).astype(np.float32) * 1e-6, a) if hasattr(a, "shape") else a
             for a in args]
    yield "small_scale", small
    large = [conv(rng.standard_normal(a.shape).astype(np.float32) * 1e6, a) if hasattr(a, "shape") else a
             for a in args]
    yield "large_scale", large


def check(baseline, candidate, input_factory, mx, enabled: set[str], n_seeds: int = 5,
          sizes=("small", "typical", "large")) -> tuple[bool, list[str]]:
    """The reference's check loop (checker.py:77-218) over an ``mx`` namespace
    (the oracle's): returns (passed, failure strings)."""
    tol = checker_tolerance(enabled)
    failures = []
    for size in sizes:
        for seed in range(n_seeds):
            args, kwargs = input_factory(size, seed)

            def as_array(v, like):
                return mx.array(v).astype(like.dtype)

            for name, vargs in edge_variants(args, seed, as_array=as_array):
                try:
                    bo = baseline(*vargs, **kwargs)
                    co = candidate(*vargs, **kwargs)
                    bl = list(bo) if isinstance(bo, (list, tuple)) else [bo]
                    cl = list(co) if isinstance(co, (list, tuple)) else [co]
                    ok, max_diff = True, 0.0
                    for b, c in zip(bl, cl):
                        is_bf16 = b.dtype.name == "bfloat16"
                        b_np = np.asarray(b).astype(np.float32) if is_bf16 else np.asarray(b)
                        c_np = np.asarray(c).astype(np.float32) if c.dtype.name == "bfloat16" else np.asarray(c)
                        v = compare_output(b_np, c_np, tol, is_bf16)
                        if not v.ok:
                            ok = False
                            max_diff = max(max_diff, v.max_diff)
                    if not ok:
                        failures.append(f"size={size} seed={seed} variant={name} max_diff={max_diff:.3e}")
                except Exception as exc:  # noqa: BLE001
                    failures.append(f"size={size} seed={seed} variant={name} exception={exc}")
    return not failures, failures
