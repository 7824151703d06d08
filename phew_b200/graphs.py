"""``mx.compile`` on B200: deferred, fused elementwise evaluation.

Stands in for the ``Compile`` node / ``@mx.compile`` decorator that
``CompileBoundaryPass`` adds (phew ``rules/compile_boundaries.py:24-48``,
``emit/codegen.py:35-49``).
"""

from __future__ import annotations

import functools


def compile_function(fn):
    """Return `fn` wrapped for ``@mx.compile``.

    Inside the wrapped call elementwise ops are deferred and fused: each
    group of elementwise ops between two other ops (a matmul, a reduction, a
    softmax, a view, ...) runs as one generated kernel, with every op rounded
    to its own dtype as op-by-op evaluation rounds it (see
    ``phew_b200.mx.core``, "deferred elementwise results").  The returned
    arrays are ordinary, materialised arrays.
    """
    from .mx import core

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        core.trace_enter()
        try:
            out = fn(*args, **kwargs)
            return core.settle(out)
        finally:
            core.trace_exit()

    wrapper.__phew_compiled__ = True
    return wrapper
