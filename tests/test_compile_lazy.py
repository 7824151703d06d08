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


def _rms_tail(core, shape, dtype=torch.bfloat16):
    x = _arr(core, shape, dtype)
    w = _arr(core, shape[-1:], dtype)
    eps = core.array._wrap(torch.tensor(1e-5, dtype=dtype))
    core.trace_enter()
    try:
        m = core.mean(x * x, axis=[len(shape) - 1], keepdims=True)
        y = x * core.rsqrt(m + eps) * w
        parts = core._fused_dag(y)
    finally:
        core.trace_exit()
    return m, y, parts


def test_keepdims_row_reduction_is_deferred(core):
    m, y, (chain, ext_specs, ext_arrays, root, key) = _rms_tail(core, (2, 3, 64))
    assert isinstance(m, core._Lazy) and m.pending and not m._pending_dag
    assert m.shape == (2, 3, 1) and m.dtype.name == "bfloat16"
    assert m._op[0] == core._ROW_REDUCE and m._op[1] == "mean"
    # the tail's DAG reads the deferred mean as an external input
    assert sum(1 for a in ext_arrays if a is m) == 1


@pytest.mark.parametrize("shape,dtype", [((8, 16, 4096), torch.bfloat16), ((3, 7, 1000), torch.float16),
                                         ((5, 256), torch.float32), ((4, 96), torch.bfloat16)])
def test_row_map_source_compiles(core, shape, dtype):
    from test_cuda_codegen import nvrtc_compile

    from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen
    from phew_b200.kernel import check_io_contract, full_source

    m, y, (chain, ext_specs, ext_arrays, root, key) = _rms_tail(core, shape, dtype)
    i = [k for k, a in enumerate(ext_arrays) if a is m][0]
    ckey, args, arrays = core._row_map_parts(y, chain, ext_specs, ext_arrays, root, key, i)
    src, ins, outs = SubgraphCUDACodegen().emit_row_map(*args)
    # x is read by both the reduction and the tail: one kernel input (x, eps, w)
    assert len(arrays) == 3 and len(ins) == 3
    assert sum(1 for a in arrays if a.shape == shape) == 1
    assert f"rowlen={shape[-1]}" in src and "phew_rowv" in src
    dts = [a.dtype.name for a in arrays]
    full = full_source("k", ins, outs, src, "", dts, [y.dtype.name])
    rc, log = nvrtc_compile(full)
    assert rc == 0, log
    check_io_contract(src, [a.shape for a in arrays], [y.shape])
    check_io_contract(src, [(11,) + shape[1:], (), shape[-1:]], [(11,) + shape[1:]])  # other row counts
    with pytest.raises(ValueError, match="rows of"):  # other row lengths are refused
        check_io_contract(src, [shape[:-1] + (shape[-1] * 2,), (), (shape[-1] * 2,)],
                          [shape[:-1] + (shape[-1] * 2,)])


def test_row_map_refuses_other_row_shapes(core):
    x = _arr(core, (4, 64))
    z = _arr(core, (2, 4, 64))
    core.trace_enter()
    try:
        m = core.mean(x * x, axis=-1, keepdims=True)
        y = z * m  # broadcasts over another leading axis: not the reduction's rows
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(y)
    finally:
        core.trace_exit()
    i = [k for k, a in enumerate(ext_arrays) if a is m][0]
    assert core._row_map_parts(y, chain, ext_specs, ext_arrays, root, key, i) is None


def test_layer_norm_fuses_the_second_reduction(core):
    """x - mean(x), then mean of its square, then the tail: the tail's DAG
    reads two deferred reductions; the variance (whose rows are the tail's)
    runs in the tail's kernel and reads the mean as an ordinary input."""
    from test_cuda_codegen import nvrtc_compile

    from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen
    from phew_b200.kernel import full_source

    x = _arr(core, (4, 9, 512))
    w = _arr(core, (512,))
    core.trace_enter()
    try:
        m = core.mean(x, axis=-1, keepdims=True)  # a plain input's reduction is deferred too
        assert isinstance(m, core._Lazy) and m._op[0] == core._ROW_REDUCE and m._op[2] is x
        d = x - m
        v = core.mean(d * d, axis=-1, keepdims=True)
        y = d * core.rsqrt(v + 1e-5) * w
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(y)
    finally:
        core.trace_exit()
    pend = [k for k, a in enumerate(ext_arrays) if isinstance(a, core._Lazy) and a.pending]
    assert [ext_arrays[k] for k in pend] == [m, v]
    parts = core._row_map_parts(y, chain, ext_specs, ext_arrays, root, key, pend[-1])
    assert parts is not None
    ckey, args, arrays = parts
    assert any(a is m for a in arrays) and not any(a is v for a in arrays)
    src, ins, outs = SubgraphCUDACodegen().emit_row_map(*args)
    full = full_source("k", ins, outs, src, "", [a.dtype.name for a in arrays], ["bfloat16"])
    rc, log = nvrtc_compile(full)
    assert rc == 0, log
    # the mean's own row map: its source (x) is a plain input, read once
    mparts = core._row_map_parts(y, chain, ext_specs, ext_arrays, root, key, pend[0])
    assert mparts is not None


def test_deferred_reduction_materialises_without_deferring_again(core, monkeypatch):
    """Reading a deferred reduction while tracing computes it (once) instead
    of deferring it again."""
    x = _arr(core, (3, 8))
    calls = []

    def fake_now(opname, a, axis, keepdims):
        calls.append((opname, a.shape, axis, keepdims))
        return core.array._wrap(torch.ones((3, 1), dtype=torch.bfloat16))

    monkeypatch.setattr(core, "_reduce_now", fake_now)
    core.trace_enter()
    try:
        m = core.max(x, axis=-1, keepdims=True)
        assert isinstance(m, core._Lazy) and m.pending
        t = m._t
    finally:
        core.trace_exit()
    assert calls == [("max", (3, 8), -1, True)]
    assert not m.pending and tuple(t.shape) == (3, 1)
    # outside tracing nothing is deferred
    core.max(x, axis=-1, keepdims=True)
    assert len(calls) == 2


def test_row_map_needs_a_shared_full_size_input(core):
    """(h @ W) * rsqrt(mean(h1 * h1) + eps): the reduction and the chain read
    different full-size arrays, so they stay two kernels."""
    h1 = _arr(core, (4, 64))
    hw = _arr(core, (4, 64))
    core.trace_enter()
    try:
        m = core.mean(h1 * h1, axis=-1, keepdims=True)
        y = hw * core.rsqrt(m + 1e-5)
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(y)
    finally:
        core.trace_exit()
    i = [k for k, a in enumerate(ext_arrays) if a is m][0]
    assert core._row_map_parts(y, chain, ext_specs, ext_arrays, root, key, i) is None


@pytest.mark.parametrize("s_shape,m_shape,groups,min_bytes", [
    ((3, 7, 256), (7, 256), (3, 7), 0),
    ((2, 4, 5, 64), (5, 64), (8, 5), 0),
    ((2, 4, 5, 64), (4, 5, 64), (2, 20), 0),
    ((3, 7, 256), (7, 256), None, 7 * 256 * 2 + 2),         # mask below the size bound
    ((3, 7, 256), (256,), None, 0),
    ((3, 7, 256), (3, 7, 256), None, 0),
    ((2, 2, 2048, 4096), (2048, 4096), (4, 2048), None),    # 16 MiB mask at the default bound
])
def test_fused_softmax_row_order(core, monkeypatch, s_shape, m_shape, groups, min_bytes):
    """softmax(s * c + mask) over the last axis: rows that read the same rows
    of a large mask are given to neighbouring blocks (position p -> row
    (p % outer) * inner + p / outer), a permutation of the rows; the source
    compiles for sm_100a."""
    from test_cuda_codegen import nvrtc_compile

    import phew_b200.emit.cuda_codegen as cg
    from phew_b200.emit.cuda_codegen import SubgraphCUDACodegen, classify_input, shared_row_groups
    from phew_b200.kernel import full_source

    if min_bytes is not None:
        monkeypatch.setattr(cg, "SHARED_ROWS_MIN_BYTES", min_bytes)

    s, m = _arr(core, s_shape), _arr(core, m_shape)
    core.trace_enter()
    try:
        chain, ext_specs, ext_arrays, root, key = core._fused_dag(s * 0.125 + m)
    finally:
        core.trace_exit()
    classes = [classify_input(tuple(x.shape), s_shape) for x in ext_specs]
    assert shared_row_groups(classes, s_shape, [2] * len(classes)) == groups
    tpr, rpb, vpt = core._softmax_row_plan(s_shape[-1], 2)
    src, ins, outs = SubgraphCUDACodegen().emit_softmax(chain, ext_specs, root, tpr, rpb, vpt)
    assert ("phew_p % " in src) == (groups is not None)
    if groups is not None:
        outer, inner = groups
        rows = outer * inner
        assert sorted((p % outer) * inner + p // outer for p in range(rows)) == list(range(rows))
    full = full_source("k", ins, outs, src, "", [a.dtype.name for a in ext_arrays], ["bfloat16"])
    rc, log = nvrtc_compile(full)
    assert rc == 0, log
