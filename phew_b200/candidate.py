"""Steps 1, 6 and 7 of phew's ``Optimizer.run`` on this backend: benchmark
the baseline, build the candidate from its ``output_source``, benchmark it
at the three problem sizes, verify it, and decide whether it is a
significant win.

The reference runs these steps inside ``Optimizer.run``
(``optimizer.py:116-126`` for the baseline benchmark, ``:290-335`` for the
candidate and ``:337-353`` for the summary), on MLX.  After
``integration.install()`` that same code reaches this backend through the
rebound ``benchmark`` / ``compare`` / ``EquivalenceChecker``; this module
states the steps on their own, so that a candidate emitted by the
reference's passes (its ``output_source``) can be judged here without the
reference's Python package: the same calls in the same order, the same
fields, the same decisions:

* a candidate that fails to build is replaced by the baseline function
  (``:293-297``);
* the speedup of every size counts; a size whose benchmark raises is
  skipped (``:303-313``);
* a candidate that fails verification is dropped: ``output_source``
  becomes the "verification failed" comment (``:318-327``);
* ``is_significant`` = verified and every size faster by more than 3 %
  (``:331-333``); a speedup under 1.05x adds the near-optimal warning.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

from .bench import benchmark, compare
from .verify import EquivalenceChecker, SubstitutionClass

DROPPED_SOURCE = "# Verification failed — no optimization applied\n"


@dataclass
class CandidateResult:
    """The fields of the reference's ``OptimizationResult`` that steps 1,
    6 and 7 produce (``optimizer.py:25-39``), plus the per-size speedups."""

    baseline_ms: float
    optimized_ms: float
    speedup: float
    is_significant: bool
    converged: bool
    verification_passed: bool
    verification_details: list = field(default_factory=list)
    search_trace: list = field(default_factory=list)
    output_source: str = ""
    warnings: list = field(default_factory=list)
    size_speedups: dict = field(default_factory=dict)


def build_fn_from_source(source: str, fn_name: str) -> Callable:
    """Compile emitted Python source and return the function
    (``optimizer.py:365-369``)."""
    ns: dict[str, Any] = {}
    exec(compile(source, "<phew_emitted>", "exec"), ns)
    return ns[fn_name]


def evaluate_candidate(
    fn: Callable,
    input_factory: Callable[[str, int], tuple[list, dict]],
    output_source: str,
    fn_name: str = "optimized",
    enabled_subst_classes: set | None = None,
) -> CandidateResult:
    """Benchmark `fn` and the candidate `output_source` defines (CUDA-event
    timing, cold L2), at the typical size and at every size, verify the
    candidate with the equivalence protocol and summarise."""
    classes = enabled_subst_classes or {SubstitutionClass.fp32_to_fp32}
    trace: list[str] = []
    warnings: list[str] = []

    trace.append("Step 1: Baseline benchmark")
    args_typical, kwargs_typical = input_factory("typical", 0)
    base = benchmark(fn, *args_typical, **kwargs_typical)
    trace.append(f"  baseline: {base.mean_ms:.3f} ± {base.std_ms:.3f} ms")
    if not base.converged:
        warnings.append("Baseline benchmark did not converge (σ/μ > 5%)")

    trace.append("Step 6: Benchmark candidate")
    try:
        optimized_fn = build_fn_from_source(output_source, fn_name)
    except Exception as exc:  # noqa: BLE001  (the reference keeps the baseline)
        warnings.append(f"Failed to build optimized fn: {exc}")
        optimized_fn = fn
    opt = benchmark(optimized_fn, *args_typical, **kwargs_typical)
    trace.append(f"  optimized: {opt.mean_ms:.3f} ± {opt.std_ms:.3f} ms")
    speedups: dict[str, float] = {}
    for size in ("small", "typical", "large"):
        try:
            args_s, kwargs_s = input_factory(size, 0)
            b = benchmark(fn, *args_s, **kwargs_s)
            o = benchmark(optimized_fn, *args_s, **kwargs_s)
            speedups[size] = b.mean_ms / o.mean_ms if o.mean_ms > 0 else 1.0
            trace.append(f"  {size}: {speedups[size]:.3f}×")
        except Exception:  # noqa: BLE001  (a size that fails is skipped, as in the reference)
            pass

    trace.append("Step 7: Equivalence verification")
    verify = EquivalenceChecker(enabled_classes=classes).check(fn, optimized_fn, input_factory)
    trace.append(f"  {verify}")
    source = output_source
    if not verify.passed:
        warnings.append("Verification FAILED — candidate dropped")
        source = DROPPED_SOURCE

    cmp = compare(base, opt)
    speedup = cmp["speedup"]
    significant = verify.passed and all(s > 1.03 for s in speedups.values())
    if speedup < 1.05 and verify.passed:
        warnings.append(f"Final speedup {speedup:.3f}× < 1.05× — input may be near-optimal.")
    return CandidateResult(
        baseline_ms=base.mean_ms, optimized_ms=opt.mean_ms, speedup=speedup,
        is_significant=significant, converged=base.converged and opt.converged,
        verification_passed=verify.passed, verification_details=list(verify.failures),
        search_trace=trace, output_source=source, warnings=warnings, size_speedups=speedups)
