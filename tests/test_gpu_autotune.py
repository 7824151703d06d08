"""Phase-2 launch search and the CUPTI profile on the device."""

from __future__ import annotations

import types

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _factory(mx, shapes):
    def f(size, seed):
        rng = np.random.default_rng(seed)
        return [mx.array(rng.standard_normal(s).astype(np.float32)) for s in shapes], {}
    return f


def test_user_kernel_keeps_its_grid_and_verifies(mx):
    from phew_b200.emit.autotune import KernelParamSearch

    src = """
    const unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < x_size) y[i] = x[i] * 2.0f;
    """
    factory = _factory(mx, [(1 << 16,)])
    x0 = factory("typical", 0)[0][0]
    node = types.SimpleNamespace(source=src, input_names=["x"], output_names=["y"],
                                 output_shapes=[x0.shape], output_dtypes=["float32"], grid=(x0.size, 1, 1),
                                 attrs={}, header="", name="double_it")
    res = KernelParamSearch(baseline_fn=lambda x: x * 2.0, max_candidates=10).search(node, factory)
    assert res and all(c.verified and c.measured_ms > 0 for c in res)
    assert all(c.grid == (x0.size, 1, 1) for c in res)
    assert res == sorted(res, key=lambda c: c.measured_ms)


def test_emitted_chain_grid_is_searched(mx):
    from phew_b200.emit.autotune import KernelParamSearch
    from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen
    from phew_b200.graph import NodeSpec

    n = 1 << 20
    x = NodeSpec("Input", (n,), "float32")
    a = NodeSpec("Input", (n,), "float32")
    m = NodeSpec("Elementwise", (n,), "float32", inputs=[x.id, a.id], op="mul")
    c = NodeSpec("Constant", (), "float32", value=1.5)
    y = NodeSpec("Elementwise", (n,), "float32", inputs=[m.id, c.id], op="add")
    src, ins, outs = SubgraphCUDACodegen().emit([m, c, y], [x, a], [y])
    node = types.SimpleNamespace(source=src, input_names=ins, output_names=outs, output_shapes=[(n,)],
                                 output_dtypes=["float32"], grid=None, attrs={}, header="", name="chain")

    def factory(size, seed):
        rng = np.random.default_rng(seed)
        return [mx.array(rng.standard_normal(n).astype(np.float32)) for _ in range(2)], {}

    res = KernelParamSearch(baseline_fn=lambda p, q: p * q + 1.5, max_candidates=12,
                            bottleneck="memory_bound").search(node, factory)
    assert res and {c.waves for c in res} <= {1, 2, 4, 8, 16}
    assert all(c.threadgroup[0] >= 128 for c in res)


def test_profile_lists_this_backends_kernels(mx):
    from phew_b200 import trace

    x = mx.array(np.random.default_rng(0).standard_normal((1024, 1024)).astype(np.float32))

    def f(x):
        return mx.softmax(x * 2.0 + 1.0, axis=-1)

    d = trace.profile(f, x)
    assert d.n_kernels >= 2 and d.total_ms > 0
    names = " ".join(k.name for k in d.kernels)
    assert "softmax" in names and "phew_ew" in names
    assert trace.classify(d).value in ("launch_overhead", "memory_bound")
