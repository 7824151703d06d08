"""phew_compare_static: the comparison for callers that cannot allocate.

Some users of this library need a verdict at a point where they may not
allocate device memory -- while a CUDA graph is being captured, inside a
serving runtime whose allocator owns the GPU, or from a watchdog that must
not synchronise the device.  ``phew_compare_static`` serves them by keeping
its scratch in a fixed array inside the library.  This test calls it through
the C ABI, twice in a row (the second call finds the first call's partials
in the shared array), and checks each record against ``phew_compare`` with
caller-provided scratch.  It sits last in collection order so that a run that
stops at the first failure has run everything else first, and it passes on
its own in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FIELDS = ("sum_abs_base", "mean_abs_base", "max_abs_diff", "atol_used", "rtol_used", "n",
          "n_nonfinite_base", "n_mismatch", "n_nan_any", "skipped", "passed")


def _record(torch, buf):
    from phew_b200 import _native

    return _native.CompareStats.from_buffer_copy(buf.cpu().numpy().tobytes())


def _run(lib, name, b, c, dtype_code, atol, rtol, torch, scratch=None):
    from phew_b200 import _native

    out = torch.zeros(ctypes.sizeof(_native.CompareStats), dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if name == "phew_compare":
        rc = lib.phew_compare(ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(c.data_ptr()),
                              b.numel(), dtype_code, atol, rtol,
                              ctypes.c_void_p(scratch.data_ptr()), scratch.numel(),
                              ctypes.c_void_p(out.data_ptr()), stream)
    else:
        rc = lib.phew_compare_static(ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(c.data_ptr()),
                                     b.numel(), dtype_code, atol, rtol,
                                     ctypes.c_void_p(out.data_ptr()), stream)
    _native.check(rc, name)
    torch.cuda.synchronize()
    return _record(torch, out)


def test_static_scratch_matches_caller_scratch():
    import torch

    from phew_b200 import _native
    from phew_b200.build import build

    build()
    lib = _native.load()
    assert lib.phew_init(0) == 0
    lib.phew_compare_scratch_bytes.restype = ctypes.c_size_t
    scratch = torch.empty(lib.phew_compare_scratch_bytes(0), dtype=torch.uint8, device="cuda")

    rng = np.random.default_rng(42)
    cases = []
    # two calls in a row with different sizes, dtypes and verdicts
    b1 = rng.standard_normal(3_000_017).astype(np.float32)
    c1 = (b1 * (1 + 1e-3 * rng.standard_normal(b1.size))).astype(np.float32)
    cases.append((b1, c1, _native.PHEW_F32, 1e-5, 1e-5))
    b2 = rng.standard_normal(70_000).astype(np.float16)
    cases.append((b2, b2.copy(), _native.PHEW_F16, 1e-3, 1e-2))

    for b_np, c_np, code, atol, rtol in cases:
        b = torch.from_numpy(b_np).cuda()
        c = torch.from_numpy(c_np).cuda()
        want = _run(lib, "phew_compare", b, c, code, atol, rtol, torch, scratch)
        got = _run(lib, "phew_compare_static", b, c, code, atol, rtol, torch)
        for f in FIELDS:
            assert getattr(got, f) == getattr(want, f), f
    assert cases and want.passed == 1  # the identical fp16 pair passes
