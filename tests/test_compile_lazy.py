"""mx.compile's deferred elementwise DAGs, built and emitted on the CPU (no
kernel runs here; tests/test_gpu_compile.py runs them)."""

from __future__ import annotations

import pytest
import torch


@pytest.fixture()
def core():
    from phew_b200.mx import core as c

    return c


def _arr(core, shape, dtype=torch.bfloat16):
    return core.array._wrap(torch.zeros(shape, dtype=dtype))


def test_elementwise_is_deferred_only_while_tracing(core):
    x = _arr(core, (4, 8))
    core.trace_enter()
    try:
        y = x * 2.0 + x
        assert isinstance(y, core._Lazy) and y.pending
        assert y.shape == (4, 8) and y.dtype.name == "bfloat16" and y.size == 32 and y.ndim == 2
    finally:
        core.trace_exit()
    assert not core._tracing()


def test_dag_structure_and_key(core):
    x0 = _arr(core, (2, 3, 16))
    t2 = _arr(core, (2, 3, 1))
    w = _arr(core, (16,))
    core.trace_enter()
    try:
        c = core.array._wrap(torch.tensor(1e-5, dtype=torch.bfloat16))
        t5 = core.rsqrt(t2 + c)
        t7 = (x0 * t5) * w
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(t7)
        # external inputs in first-visit order, each once
        assert [a is b for a, b in zip(ext_arrays, [x0, t2, c, w])] == [True] * 4
        assert [n.kind for n in chain].count("Elementwise") == 4
        assert root is chain[-1] and root.shape == (2, 3, 16)
        # the same structure over other arrays gives the same key (kernel reuse)
        y0, y2, v = _arr(core, (2, 3, 16)), _arr(core, (2, 3, 1)), _arr(core, (16,))
        t7b = (y0 * core.rsqrt(y2 + c)) * v
        assert core._fused_dag(t7b)[-1] == key
        # a different scalar is a different kernel
        t7c = (y0 * core.rsqrt(y2 + c)) * 3.0
        assert core._fused_dag(t7c)[-1] != key
    finally:
        core.trace_exit()


def test_shared_subexpression_visited_once(core):
    x = _arr(core, (8,))
    core.trace_enter()
    try:
        t = x + 1.0
        y = t * t
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(y)
        assert len(ext_arrays) == 1
        assert [n.kind for n in chain].count("Elementwise") == 2
    finally:
        core.trace_exit()


def test_mixed_dtypes_insert_casts(core):
    a = _arr(core, (8,), torch.float16)
    b = _arr(core, (8,), torch.float32)
    core.trace_enter()
    try:
        y = a + b
        assert y.dtype.name == "float32"
        chain = core._fused_dag(y)[0]
        assert [n.kind for n in chain] == ["Cast", "Elementwise"]
    finally:
        core.trace_exit()


def test_fused_source_emits_one_kernel(core):
    from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen

    s = _arr(core, (2, 4, 64, 64))
    mask = _arr(core, (64, 64))
    core.trace_enter()
    try:
        y = s * 0.08838834764831843 + mask
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(y)
    finally:
        core.trace_exit()
    src, ins, outs = SubgraphCUDACodegen().emit(chain, ext_specs, [root])
    assert len(ins) == 2 and len(outs) == 1
    assert "inp1=suffix:4096" in src


def test_compile_wrapper_returns_plain_arrays_and_restores_state(core):
    from phew_b200.graphs import compile_function

    calls = []

    def f(x):
        calls.append(core._tracing())
        return [x, (x, {"k": x})]

    g = compile_function(f)
    x = _arr(core, (3,))
    out = g(x)
    assert calls == [True] and not core._tracing()
    assert out[0] is x and out[1][1]["k"] is x

    def bad(x):
        raise RuntimeError("boom")

    with pytest.raises(RuntimeError):
        compile_function(bad)(x)
    assert not core._tracing()


def test_dag_walk_leaves_no_reference_cycle(core):
    """Arrays reached while fusing must be freed by reference counting alone
    (the cyclic collector does not run on device-memory pressure)."""
    import gc
    import weakref

    x = _arr(core, (16,))
    ref = weakref.ref(x._t)
    core.trace_enter()
    try:
        y = x * 2.0 + 1.0
        core._fused_dag(y)
    finally:
        core.trace_exit()
    gc.disable()
    try:
        del x, y
        assert ref() is None
    finally:
        gc.enable()
