"""Substitution classes and tolerances (phew ``verify/tolerances.py:12-36``).

Same names, values and opt-in flags as the reference, so verdicts are
computed against identical thresholds.  Members compare equal by value to
phew's own ``SubstitutionClass`` through :func:`as_subst_class`.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class SubstitutionClass(Enum):
    fp32_to_fp32 = "fp32_to_fp32"
    fp32_to_fp16 = "fp32_to_fp16"
    fp32_to_bf16 = "fp32_to_bf16"
    quantized_4bit = "quantized_4bit"
    normed_matmul = "normed_matmul"


@dataclass(frozen=True)
class Tolerance:
    atol: float
    rtol: float
    opt_in: bool


TOLERANCES: dict[SubstitutionClass, Tolerance] = {
    SubstitutionClass.fp32_to_fp32: Tolerance(atol=1e-5, rtol=1e-5, opt_in=False),
    SubstitutionClass.fp32_to_fp16: Tolerance(atol=1e-3, rtol=1e-2, opt_in=True),
    SubstitutionClass.fp32_to_bf16: Tolerance(atol=1e-2, rtol=1e-2, opt_in=True),
    SubstitutionClass.quantized_4bit: Tolerance(atol=1e-2, rtol=5e-2, opt_in=True),
    SubstitutionClass.normed_matmul: Tolerance(atol=1e-3, rtol=1e-1, opt_in=True),
}


def as_subst_class(c) -> SubstitutionClass:
    """Accept this module's enum, phew's enum (same values) or a string."""
    if isinstance(c, SubstitutionClass):
        return c
    return SubstitutionClass(getattr(c, "value", c))
