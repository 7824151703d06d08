"""``mx.compile`` on B200: capture a function's launches in a CUDA graph.

Stands in for the ``Compile`` node / ``@mx.compile`` decorator that
``CompileBoundaryPass`` adds (phew ``rules/compile_boundaries.py:24-48``,
``emit/codegen.py:35-49``).
"""

from __future__ import annotations

import functools


def compile_function(fn):
    """Return `fn` wrapped for ``@mx.compile`` (eager execution for now)."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        return fn(*args, **kwargs)

    wrapper.__phew_compiled__ = True
    return wrapper
