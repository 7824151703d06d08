"""Convergence rule of the search loop (phew ``bench/convergence.py:11-25``).

A candidate wins only if it is more than 3% faster and beats the current best
on every problem size tested.
"""

from __future__ import annotations

IMPROVEMENT_THRESHOLD = 0.03


def check_convergence(
    current_best_ms: float,
    candidate_ms: float,
    problem_sizes: int = 1,
    problems_beaten: int = 0,
) -> bool:
    if current_best_ms <= 0:
        return False
    speedup = current_best_ms / candidate_ms
    return speedup > (1.0 + IMPROVEMENT_THRESHOLD) and problems_beaten >= problem_sizes
