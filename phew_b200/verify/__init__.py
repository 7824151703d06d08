from .checker import N_SEEDS, PROBLEM_SIZES, EquivalenceChecker, VerificationResult, compare_arrays
from .tolerances import TOLERANCES, SubstitutionClass, Tolerance

__all__ = [
    "EquivalenceChecker",
    "VerificationResult",
    "compare_arrays",
    "SubstitutionClass",
    "Tolerance",
    "TOLERANCES",
    "N_SEEDS",
    "PROBLEM_SIZES",
]
