from .convergence import check_convergence
from .harness import BenchResult, benchmark, compare

__all__ = ["BenchResult", "benchmark", "compare", "check_convergence"]
