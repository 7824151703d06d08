"""Equivalence checker with device-side comparison.

Same protocol and verdict rule as phew's ``EquivalenceChecker``
(``verify/checker.py:46-263``): for size in small/typical/large, for seed in
0..n_seeds-1, for each edge variant (random, zeros, x1e-6, x1e6 drawn from
``np.random.default_rng(seed + 1000)``), run baseline and candidate, and
compare every output pair with the allclose rule (NaN positions must agree;
non-finite baselines and extreme bf16 outputs are skipped; bf16 outputs get
the output-scale-relative tolerance).  One failing unit fails the candidate.

The comparison itself runs on the GPU (``phew_compare``): each output is read
once from HBM and only a 64-byte record comes back to the host.  Outputs of
non-float dtypes are compared on the host with numpy, as the reference does.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np
import torch

from .. import _native
from .tolerances import TOLERANCES, SubstitutionClass, Tolerance, as_subst_class

N_SEEDS = 5
PROBLEM_SIZES = ["small", "typical", "large"]


@dataclass
class VerificationResult:
    passed: bool
    substitution_class: SubstitutionClass
    tolerance: Tolerance
    seeds_tested: int
    sizes_tested: list[str]
    failures: list[str] = field(default_factory=list)
    details: dict[str, Any] = field(default_factory=dict)

    def __str__(self) -> str:
        status = "PASS" if self.passed else "FAIL"
        return (
            f"[{status}] {self.substitution_class.value} "
            f"atol={self.tolerance.atol} rtol={self.tolerance.rtol} "
            f"seeds={self.seeds_tested} sizes={self.sizes_tested}"
            + (f" failures={self.failures}" if self.failures else "")
        )


class _CompareBuffers:
    """Per-device scratch and result record for phew_compare."""

    def __init__(self, dev: torch.device) -> None:
        lib = _native.load()
        lib.phew_compare_scratch_bytes.restype = ctypes.c_size_t
        self.scratch_bytes = int(lib.phew_compare_scratch_bytes(0))
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=dev)
        self.record = torch.empty(ctypes.sizeof(_native.CompareStats), dtype=torch.uint8, device=dev)


_buffers: dict[int, _CompareBuffers] = {}

# Bytes of comparison records read back to the host so far (one record per
# compared output): what a verification run moves device -> host.
readback_bytes = 0


def _bufs(dev: torch.device) -> _CompareBuffers:
    b = _buffers.get(dev.index)
    if b is None:
        b = _CompareBuffers(dev)
        _buffers[dev.index] = b
    return b


def compare_arrays(b, c, atol: float, rtol: float) -> _native.CompareStats:
    """Run the allclose rule of the reference on device arrays b (baseline)
    and c (candidate) of the same shape; returns the comparison record."""
    from ..dtypes import float32
    from ..mx.core import asarray_device, astype

    b = asarray_device(b)
    c = asarray_device(c)
    if b.shape != c.shape:
        raise ValueError(f"output shapes differ: baseline {b.shape} vs candidate {c.shape}")
    if c.dtype is not b.dtype:
        # numpy would compare in the promoted dtype
        from ..dtypes import promote

        p = promote(b.dtype, c.dtype)
        b, c = astype(b, p), astype(c, p)
    if b.dtype.code is None:
        raise TypeError("compare_arrays: non-float outputs are compared on the host")
    bufs = _bufs(b._t.device)
    _native.call(
        "phew_compare",
        ctypes.c_void_p(b._t.data_ptr()),
        ctypes.c_void_p(c._t.data_ptr()),
        ctypes.c_int64(b.size),
        b.dtype.code,
        ctypes.c_double(atol),
        ctypes.c_double(rtol),
        ctypes.c_void_p(bufs.scratch.data_ptr()),
        ctypes.c_size_t(bufs.scratch_bytes),
        ctypes.c_void_p(bufs.record.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    raw = bufs.record.cpu().numpy().tobytes()
    global readback_bytes
    readback_bytes += len(raw)
    _ = float32  # keep the import local to the device path
    return _native.CompareStats.from_buffer_copy(raw)


def _host_compare(b_np: np.ndarray, c_np: np.ndarray, tol: Tolerance) -> tuple[bool, float]:
    if not np.all(np.isfinite(b_np.astype(np.float64))):
        return True, 0.0
    nan_match = np.isnan(b_np.astype(np.float64)) == np.isnan(c_np.astype(np.float64))
    close = np.isclose(b_np, c_np, atol=tol.atol, rtol=tol.rtol)
    ok = bool(np.all(nan_match & close))
    if ok:
        return True, 0.0
    return False, float(np.max(np.abs(b_np.astype(np.float64) - c_np.astype(np.float64))))


class EquivalenceChecker:
    """Verify that two callables are equivalent under a substitution class."""

    def __init__(
        self,
        subst_class: Any = SubstitutionClass.fp32_to_fp32,
        n_seeds: int = N_SEEDS,
        enabled_classes: set | None = None,
        problem_sizes: list[str] | None = None,
    ) -> None:
        self.subst_class = as_subst_class(subst_class)
        self.n_seeds = n_seeds
        if enabled_classes is None:
            enabled_classes = {SubstitutionClass.fp32_to_fp32}
        self.enabled_classes = {as_subst_class(c) for c in enabled_classes}
        self.problem_sizes = list(problem_sizes or PROBLEM_SIZES)
        self.tolerance = max(
            (TOLERANCES[c] for c in self.enabled_classes if c in TOLERANCES),
            key=lambda t: t.atol,
            default=TOLERANCES[SubstitutionClass.fp32_to_fp32],
        )

    # -- one verification unit ---------------------------------------------------
    def check_unit(self, out_baseline, out_candidate) -> tuple[bool, float]:
        """Compare one (baseline, candidate) output set; returns (ok, max_diff)."""
        from ..dtypes import bfloat16
        from ..mx.core import array

        b_outs = list(out_baseline) if isinstance(out_baseline, (list, tuple)) else [out_baseline]
        c_outs = list(out_candidate) if isinstance(out_candidate, (list, tuple)) else [out_candidate]
        ok = True
        max_diff = 0.0
        for b_arr, c_arr in zip(b_outs, c_outs):
            if not isinstance(b_arr, array) or not isinstance(c_arr, array):
                b_np, c_np = np.asarray(b_arr), np.asarray(c_arr)
                good, diff = _host_compare(b_np, c_np, self.tolerance)
            elif b_arr.dtype.code is None or c_arr.dtype.code is None:
                good, diff = _host_compare(np.asarray(b_arr), np.asarray(c_arr), self.tolerance)
            else:
                st = compare_arrays(b_arr, c_arr, self.tolerance.atol, self.tolerance.rtol)
                good = bool(st.passed)
                diff = float("nan") if st.n_nan_any > 0 else float(st.max_abs_diff)
                _ = bfloat16
            if not good:
                ok = False
                # Python max() keeps the running value when diff is NaN, as
                # the reference's loop does.
                max_diff = max(max_diff, diff)
        return ok, max_diff

    def check(
        self,
        baseline: Callable,
        candidate: Callable,
        input_factory: Callable[[str, int], tuple[list, dict]],
    ) -> VerificationResult:
        if self.subst_class not in self.enabled_classes:
            return VerificationResult(
                passed=False,
                substitution_class=self.subst_class,
                tolerance=self.tolerance,
                seeds_tested=0,
                sizes_tested=[],
                failures=[f"{self.subst_class.value} requires opt-in"],
            )
        failures: list[str] = []
        sizes_tested: list[str] = []
        for size_label in self.problem_sizes:
            sizes_tested.append(size_label)
            for seed in range(self.n_seeds):
                args, kwargs = input_factory(size_label, seed)
                for variant_name, v_args, v_kwargs in edge_variants(args, kwargs, seed):
                    try:
                        ok, max_diff = self.check_unit(baseline(*v_args, **v_kwargs),
                                                       candidate(*v_args, **v_kwargs))
                        if not ok:
                            failures.append(
                                f"size={size_label} seed={seed} variant={variant_name} "
                                f"max_diff={max_diff:.3e}"
                            )
                    except Exception as exc:  # noqa: BLE001  (reference records any failure)
                        failures.append(
                            f"size={size_label} seed={seed} variant={variant_name} exception={exc}"
                        )
        return VerificationResult(
            passed=len(failures) == 0,
            substitution_class=self.subst_class,
            tolerance=self.tolerance,
            seeds_tested=self.n_seeds,
            sizes_tested=sizes_tested,
            failures=failures,
        )


def edge_variants(args, kwargs, seed: int):
    """(name, args, kwargs) for random / zeros / small_scale / large_scale,
    drawn exactly as the reference does (``verify/checker.py:235-263``)."""
    from ..mx.core import array, zeros_like

    yield "random", args, kwargs
    yield "zeros", [zeros_like(a) if hasattr(a, "shape") else a for a in args], kwargs
    rng = np.random.default_rng(seed + 1000)
    small = [
        array(rng.standard_normal(a.shape).astype(np.float32) * 1e-6).astype(a.dtype)
        if hasattr(a, "shape") else a
        for a in args
    ]
    yield "small_scale", small, kwargs
    large = [
        array(rng.standard_normal(a.shape).astype(np.float32) * 1e6).astype(a.dtype)
        if hasattr(a, "shape") else a
        for a in args
    ]
    yield "large_scale", large, kwargs
