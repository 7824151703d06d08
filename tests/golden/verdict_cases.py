"""Verification cases whose verdicts are pinned against the reference.

Each case is (name, subst classes enabled, make(mx) -> (baseline, candidate),
input_factory(mx)).  Functions use only operations whose results are exactly
rounded on every backend (add, mul by constants), so the outputs -- and hence
the verdicts and max_diff strings -- are identical on the reference's checker
(run over the oracle namespace) and on the device checker.
"""

from __future__ import annotations

import ml_dtypes
import numpy as np

BF16 = np.dtype(ml_dtypes.bfloat16)

SIZES = {"small": (8, 16), "typical": (16, 32), "large": (32, 64)}


def _factory(mx, dtype, n_args=1):
    def f(size, seed):
        rng = np.random.default_rng(seed)
        shape = SIZES[size]
        args = [mx.array(rng.standard_normal(shape).astype(np.float32).astype(dtype))
                for _ in range(n_args)]
        return args, {}
    return f


def _same(mx):
    return (lambda x: x * 2.0 + 1.0), (lambda x: x * 2.0 + 1.0)


def _shifted(delta):
    def make(mx):
        return (lambda x: x * 2.0), (lambda x: x * 2.0 + delta)
    return make


def _scaled(f):
    def make(mx):
        return (lambda x: x * 3.0), (lambda x: x * (3.0 * f))
    return make


def _nan_candidate(mx):
    return (lambda x: x + 1.0), (lambda x: x * 0.0 + (x - x) / (x - x))


def _two_outputs(mx):
    return (lambda x, y: (x + y, x * y)), (lambda x, y: (y + x, x * y * 1.0009765625))


CASES = [
    ("fp32_identical", ["fp32_to_fp32"], _same, np.float32, 1),
    ("fp32_shift_1e-3", ["fp32_to_fp32"], _shifted(1e-3), np.float32, 1),
    ("fp32_shift_1e-9", ["fp32_to_fp32"], _shifted(1e-9), np.float32, 1),
    ("fp32_scale_1e-4", ["fp32_to_fp32"], _scaled(1.0001), np.float32, 1),
    ("fp16_identical", ["fp32_to_fp32"], _same, np.float16, 1),
    ("fp16_shift", ["fp32_to_fp32"], _shifted(2e-3), np.float16, 1),
    ("fp16_opt_in_shift", ["fp32_to_fp32", "fp32_to_fp16"], _shifted(2e-3), np.float16, 1),
    ("bf16_scale_3pct", ["fp32_to_fp32"], _scaled(1.03), BF16, 1),
    ("bf16_scale_12pct", ["fp32_to_fp32"], _scaled(1.125), BF16, 1),
    ("nan_candidate", ["fp32_to_fp32"], _nan_candidate, np.float32, 1),
    ("two_outputs_fp32", ["fp32_to_fp32"], _two_outputs, np.float32, 2),
    ("two_outputs_normed", ["fp32_to_fp32", "normed_matmul"], _two_outputs, np.float32, 2),
]


def build(case, mx):
    name, classes, make, dtype, n_args = case
    base, cand = make(mx)
    return name, classes, base, cand, _factory(mx, dtype, n_args)
