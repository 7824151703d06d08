"""tcgen05 GEMM parity against a float32 numpy product (the oracle's matmul),
covering both B layouts, ragged edges, batching, broadcasting and the fused
normed-matmul row scale."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import mlx_cpu

pytestmark = pytest.mark.gpu

BF16 = mlx_cpu.BF16


def _rand(rng, shape, dtype, scale=1.0):
    return (rng.standard_normal(shape).astype(np.float32) * scale).astype(dtype)


def check(got, ref, dtype):
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    assert g.shape == r.shape, (g.shape, r.shape)
    scale = np.sqrt(np.mean(r * r)) + 1e-30
    tol = 1e-5 if dtype == np.float32 else 2e-2
    np.testing.assert_allclose(g, r, rtol=tol, atol=tol * scale)
    # error in units of the output scale should be near the rounding level
    rel = np.abs(g - r).max() / scale
    assert rel < (1e-5 if dtype == np.float32 else 1.6e-2), rel


def check_ulps(got, ref, dtype, max_ulps=1):
    """16-bit products: both sides round an fp32 sum, so they differ by at
    most one unit in the last place of the output (fp32 sums in a different
    order straddle a rounding boundary); more means a wrong element.  Outputs
    far below the typical magnitude (sums that cancel) are held to the unit
    of 1/64 of it, where fp32 summation order shows."""
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    assert g.shape == r.shape, (g.shape, r.shape)
    mant = 7 if dtype is BF16 else 10
    floor = np.sqrt(np.mean(r * r)) / 64 + 1e-30
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(r), floor))) - mant)
    err = np.abs(g - r) / ulp
    assert err.max() <= max_ulps, (err.max(), np.unravel_index(err.argmax(), err.shape))


@pytest.fixture(autouse=True)
def _no_device_errors(mx):
    from phew_b200.ops import check_device_errors

    yield
    mx.synchronize()
    check_device_errors()


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 4096), (300, 200, 96),
                                   (1, 256, 128), (129, 257, 200), (64, 1024, 64)])
def test_gemm_b_row_major(mx, dtype, M, N, K):
    rng = np.random.default_rng(M * 7 + N)
    a = _rand(rng, (M, K), dtype)
    b = _rand(rng, (K, N), dtype, 1 / np.sqrt(K))
    got = mx.array(a) @ mx.array(b)
    check(got, mlx_cpu.matmul(mlx_cpu.array(a), mlx_cpu.array(b)), dtype)


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (512, 384, 256), (77, 130, 64)])
def test_gemm_b_transposed_view(mx, dtype, M, N, K):
    """q @ k.T: B is a transposed view of a [N, K] array (K-major operand)."""
    rng = np.random.default_rng(N)
    a = _rand(rng, (M, K), dtype)
    bt = _rand(rng, (N, K), dtype, 1 / np.sqrt(K))
    got = mx.array(a) @ mx.array(bt).T
    check(got, mlx_cpu.matmul(mlx_cpu.array(a), mlx_cpu.array(bt).T), dtype)


def test_gemm_k_transposed_from_fused_qkv(mx):
    """q @ k^T with q, k sliced out of a fused qkv projection
    (qkv.reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)): the batch dims of
    k^T do not collapse to one stride, so k is copied in its own layout and
    the GEMM reads it K-major."""
    rng = np.random.default_rng(21)
    B, T, H, D = 2, 256, 3, 128
    qkv = _rand(rng, (B, T, 3 * H * D), BF16)
    x = mx.array(qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    q, k = x[0], x[1]
    got = q @ k.transpose(0, 1, 3, 2)
    o = mlx_cpu.array(qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    ref = mlx_cpu.matmul(o[0], o[1].transpose(0, 1, 3, 2))
    check(got, ref, BF16)


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("B,T,H", [(2, 256, 3), (2, 1024, 80)])
def test_gemm_reads_fused_qkv_in_place(mx, dtype, B, T, H):
    """q @ k^T and p @ v with q, k, v (batch, head) views of a fused qkv
    projection: phew_gemm_batched2 reads them through 4-D maps, no copy (the
    larger case also takes the resident-B mode); checked on a sample of
    (batch, head) entries."""
    from phew_b200 import _native

    D = 128
    rng = np.random.default_rng(T + H)
    qkv = _rand(rng, (B, T, 3 * H * D), dtype)
    x = mx.array(qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    q, k, v = x[0], x[1], x[2]
    n0 = _native.launch_count()
    s = q @ k.transpose(0, 1, 3, 2)
    p = (s * 0.01).astype(getattr(mx, "bfloat16" if dtype is BF16 else "float16"))
    o = p @ v
    mx.synchronize()
    assert _native.launch_count() - n0 <= 4  # two GEMMs and the scale, no copies
    o_ref = mlx_cpu.array(qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    s_np, o_np, p_np = np.asarray(s), np.asarray(o), np.asarray(p)
    for b, h in sorted({(0, 0), (B - 1, H - 1), (B // 2, H // 2), (0, H - 1)}):
        qb = np.asarray(o_ref[0])[b, h]
        kb = np.asarray(o_ref[1])[b, h]
        vb = np.asarray(o_ref[2])[b, h]
        check_ulps(s_np[b, h], mlx_cpu.matmul(mlx_cpu.array(qb), mlx_cpu.array(np.ascontiguousarray(kb.T))),
                   dtype)
        check_ulps(o_np[b, h], mlx_cpu.matmul(mlx_cpu.array(p_np[b, h]), mlx_cpu.array(vb)), dtype)


def test_gemm_batched_attention_shapes(mx):
    rng = np.random.default_rng(3)
    B, H, L, D = 2, 3, 256, 128
    q = _rand(rng, (B, H, L, D), BF16)
    k = _rand(rng, (B, H, L, D), BF16)
    v = _rand(rng, (B, H, L, D), BF16)
    s = mx.array(q) @ mx.array(k).transpose(0, 1, 3, 2)
    check(s, mlx_cpu.matmul(mlx_cpu.array(q), mlx_cpu.array(k).transpose(0, 1, 3, 2)), BF16)
    p = _rand(rng, (B, H, L, L), BF16, 0.05)
    o = mx.array(p) @ mx.array(v)
    check(o, mlx_cpu.matmul(mlx_cpu.array(p), mlx_cpu.array(v)), BF16)


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("batch,M,N,K,kmajor", [(80, 1024, 1024, 128, True),    # q @ k^T, as attention
                                                (40, 1100, 2000, 64, False),    # ragged edges, B row-major
                                                (300, 1024, 300, 96, True),     # K tail, 2 column blocks
                                                (400, 1024, 128, 128, False)])  # 128-column tiles
def test_gemm_resident_b(mx, dtype, batch, M, N, K, kmajor):
    """K <= 128 with many column runs: each CTA keeps a run's B block in
    shared memory and walks the run's row blocks (checked on a sample of
    batch entries, the first and last among them)."""
    rng = np.random.default_rng(batch + M + K)
    a = _rand(rng, (batch, M, K), dtype)
    if kmajor:
        bt = _rand(rng, (batch, N, K), dtype, 1 / np.sqrt(K))
        got = mx.array(a) @ mx.array(bt).transpose(0, 2, 1)
    else:
        b = _rand(rng, (batch, K, N), dtype, 1 / np.sqrt(K))
        got = mx.array(a) @ mx.array(b)
    g = np.asarray(got)
    for i in sorted({0, 1, batch // 3, batch // 2 + 1, batch - 2, batch - 1}):
        bi = bt[i].T if kmajor else b[i]
        check(g[i], mlx_cpu.matmul(mlx_cpu.array(a[i]), mlx_cpu.array(np.ascontiguousarray(bi))), dtype)


def test_gemm_broadcast_weight(mx):
    rng = np.random.default_rng(4)
    x = _rand(rng, (3, 100, 256), BF16)
    w = _rand(rng, (256, 384), BF16, 1 / 16)
    got = mx.array(x) @ mx.array(w)
    check(got, mlx_cpu.matmul(mlx_cpu.array(x), mlx_cpu.array(w)), BF16)


def test_gemm_simt_paths(mx):
    rng = np.random.default_rng(5)
    a = _rand(rng, (33, 100), np.float32)
    b = _rand(rng, (100, 17), np.float32)
    check(mx.array(a) @ mx.array(b), mlx_cpu.matmul(mlx_cpu.array(a), mlx_cpu.array(b)), np.float32)
    a16 = _rand(rng, (40, 100), BF16)  # 100 * 2 bytes is not a multiple of 16
    b16 = _rand(rng, (100, 24), BF16, 0.1)
    check(mx.array(a16) @ mx.array(b16), mlx_cpu.matmul(mlx_cpu.array(a16), mlx_cpu.array(b16)), BF16)


def test_gemm_vector_operands(mx):
    rng = np.random.default_rng(6)
    a = _rand(rng, (128,), BF16)
    b = _rand(rng, (128, 64), BF16, 0.1)
    got = mx.array(a) @ mx.array(b)
    assert got.shape == (64,)
    check(got, mlx_cpu.matmul(mlx_cpu.array(a), mlx_cpu.array(b)), BF16)


@pytest.mark.parametrize("M,K,N", [(256, 4096, 512), (200, 512, 256), (128, 256, 128)])
def test_fused_row_sum_of_squares(mx, M, K, N):
    """The in-kernel sum of squares of each A row (row_scale mode 2)."""
    from phew_b200.ops import matmul

    rng = np.random.default_rng(M + K)
    x = _rand(rng, (M, K), BF16)
    w = _rand(rng, (K, N), BF16, 1 / np.sqrt(K))
    got = np.asarray(matmul(mx.array(x), mx.array(w), row_scale=2)).astype(np.float64)
    ss = np.sum(x.astype(np.float64) ** 2, -1)
    rel = np.abs(got[:, 0] / ss - 1)
    bad = np.nonzero(rel > 1e-2)[0]
    assert len(bad) == 0, f"rows {bad[:16]}: got {got[bad[:4], 0]} want {ss[bad[:4]]}"


@pytest.mark.parametrize("M,K,N", [(256, 4096, 512), (200, 512, 256)])
def test_normed_matmul_fused(mx, M, K, N):
    from phew_b200.ops import normed_matmul

    rng = np.random.default_rng(M)
    x = _rand(rng, (M, K), BF16)
    w = _rand(rng, (K, N), BF16, 1 / np.sqrt(K))
    got = normed_matmul(mx.array(x), mx.array(w), eps=1e-5)
    xf = x.astype(np.float32)
    r = 1.0 / np.sqrt(np.mean(xf.astype(np.float64) ** 2, -1, keepdims=True) + 1e-5)
    mm = xf @ w.astype(np.float32)
    ref = mm * r
    g = np.asarray(got).astype(np.float64)
    implied = np.sum(g * mm, -1) / np.sum(mm * mm, -1)
    bad = np.nonzero(np.abs(implied / r[:, 0] - 1) > 5e-3)[0]
    assert len(bad) == 0, f"rows with a wrong scale: {bad[:20]} ratios {(implied / r[:, 0])[bad[:8]]}"
    check(got, ref.astype(BF16), BF16)


def test_normed_matmul_in_a_cuda_graph(mx):
    """The row-factor pass, its stream-ordered workspace and the dependent
    GEMM launch are captured into a CUDA graph and replayed; replays on new
    inputs give the eager results."""
    import torch

    from phew_b200.ops import normed_matmul

    rng = np.random.default_rng(77)
    M, K, N = 512, 1024, 768
    xs = [_rand(rng, (M, K), BF16) for _ in range(2)]
    w = _rand(rng, (K, N), BF16, 1 / np.sqrt(K))
    xd, wd = mx.array(xs[0]), mx.array(w)
    eager = [np.asarray(normed_matmul(mx.array(x), wd, eps=1e-5)).view(np.uint16) for x in xs]
    normed_matmul(xd, wd, eps=1e-5)  # warm up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = normed_matmul(xd, wd, eps=1e-5)
    for x, want in zip(xs, eager):
        xd._t.copy_(torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(xd._t.device))
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(np.asarray(out).view(np.uint16), want)
    del g


@pytest.mark.parametrize("M,N,K,batch", [(8192, 4096, 1024, 1), (8192 - 64, 4096, 640, 1), (4096, 4096, 1024, 2)])
def test_gemm_last_round_as_half_tiles(mx, M, N, K, batch):
    """Shapes with 512 tiles of 256 rows on a 148-SM B200: the last, partial
    round runs as 128-row half tiles (a partial last row block and a batched
    case included); every output row must still be computed once."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(M + K)
    a = torch.randn(batch, M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    b = (torch.randn(batch, K, N, device="cuda", dtype=torch.bfloat16, generator=g) / K ** 0.5)
    got = (mx.array(a) @ mx.array(b))._t.float()
    want = a.float() @ b.float()
    err = ((got - want).abs().amax(dim=-1) / want.abs().amax(dim=-1)).max().item()
    assert err < 1e-2, err
    # rows of the half tiles at the end were written (no stale rows)
    assert torch.isfinite(got).all()


def test_normed_matmul_last_round_as_half_tiles(mx):
    from phew_b200.ops import normed_matmul

    rng = np.random.default_rng(91)
    M, K, N = 8192, 1024, 4096
    x = _rand(rng, (M, K), BF16)
    w = _rand(rng, (K, N), BF16, 1 / np.sqrt(K))
    got = np.asarray(normed_matmul(mx.array(x), mx.array(w), eps=1e-5)).astype(np.float32)
    xf = x.astype(np.float32)
    r = 1.0 / np.sqrt(np.mean(xf.astype(np.float64) ** 2, -1, keepdims=True) + 1e-5)
    want = (xf @ w.astype(np.float32)) * r
    err = np.max(np.abs(got - want).max(-1) / np.abs(want).max(-1))
    assert err < 1e-2, err
