"""Parity at the exact shapes the benchmark times.

The timed launches have grids that small-shape tests never reach: the causal
attention launch over (4, 32, 2048, 128) schedules 1024 CTAs in eight groups
of 16 heads with the longest query blocks first, and the normed matmul over
8192 x 4096 x 4096 walks 512 tiles of 256 x 256 whose last, partial round
runs as 128-row half tiles.  These tests run those launches on the
benchmark's own inputs (``phew_b200.workloads``, seed 0) and compare sampled
heads / rows with the oracle (``oracle/mlx_cpu.py``), so a scheduling or
tile-edge fault at full size is caught without a full CPU evaluation.

Tolerance: 2e-2 relative for bf16 outputs, measured against the output's
own scale (attention: the scale of V, see ``test_gpu_sdpa.check``).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import mlx_cpu

pytestmark = pytest.mark.gpu

BF16 = mlx_cpu.BF16


@pytest.fixture(autouse=True)
def _no_device_errors(mx):
    from phew_b200.ops import check_device_errors

    yield
    mx.synchronize()
    check_device_errors()


def _attention_heads(bh_total: int, group: int = 16) -> list[int]:
    """One (batch, head) index from every group of 16 the kernel schedules
    together (a different position in each group), plus the very last one."""
    picks = [g * group + (5 * g + 3) % group for g in range(bh_total // group)]
    return sorted(set(picks + [0, bh_total - 1]))


@pytest.mark.parametrize("causal", [True, False])
def test_sdpa_at_benchmark_shape(mx, causal):
    from phew_b200.workloads import ATTN_D, attention_inputs

    q, k, v, _ = attention_inputs("typical", 0)
    B, H, L, D = q.shape
    assert (B, H, L, D) == (4, 32, 2048, ATTN_D)
    scale = 1.0 / math.sqrt(D)
    mask = "causal" if causal else None
    got = np.asarray(mx.fast.scaled_dot_product_attention(
        mx.array(q), mx.array(k), mx.array(v), scale=scale, mask=mask))
    got = got.reshape(B * H, L, D)
    qf, kf, vf = (a.reshape(B * H, 1, L, D) for a in (q, k, v))
    vscale = float(np.sqrt(np.mean(vf.astype(np.float64) ** 2)))
    heads = _attention_heads(B * H)
    assert len(heads) >= 9
    for bh in heads:
        ref = mlx_cpu.sdpa(mlx_cpu.array(qf[bh:bh + 1]), mlx_cpu.array(kf[bh:bh + 1]),
                           mlx_cpu.array(vf[bh:bh + 1]), scale, mask)
        r = np.asarray(ref).astype(np.float64)[0, 0]
        g = got[bh].astype(np.float64)
        err = np.abs(g - r)
        # whole head: every query block, the first and the last causal one included
        assert np.isfinite(g).all(), bh
        assert err.max() / vscale < 2e-2, (bh, err.max() / vscale, np.unravel_index(err.argmax(), err.shape))
        np.testing.assert_allclose(g, r, rtol=2e-2, atol=2e-2 * vscale)


def _normed_rows(M: int, tile: int = 256) -> list[int]:
    """Two rows in every 256-row block, one in each 128-row half (so both
    halves of every tile are seen, whichever of them ran as a half tile),
    plus the first and last rows."""
    rows = []
    for rb in range(M // tile):
        rows.append(rb * tile + (37 * rb + 5) % 128)
        rows.append(rb * tile + 128 + (53 * rb + 11) % 128)
    return sorted(set(rows + [0, M - 1]))


def test_normed_matmul_at_benchmark_shape(mx):
    from phew_b200.ops import normed_matmul
    from phew_b200.workloads import normed_matmul_inputs

    x, w = normed_matmul_inputs("typical", 0)
    M, K = x.shape
    N = w.shape[1]
    assert (M, K, N) == (8192, 4096, 4096)
    got = np.asarray(normed_matmul(mx.array(x), mx.array(w), eps=1e-5))
    rows = _normed_rows(M)
    assert len(rows) >= 64
    xf = x[rows].astype(np.float32)
    r = 1.0 / np.sqrt(np.mean(xf.astype(np.float64) ** 2, -1, keepdims=True) + 1e-5)
    ref = ((xf @ w.astype(np.float32)) * r).astype(BF16).astype(np.float64)
    g = got[rows].astype(np.float64)
    scale = float(np.sqrt(np.mean(ref * ref)))
    # every column of each sampled row: all 16 column tiles of its row block
    np.testing.assert_allclose(g, ref, rtol=2e-2, atol=2e-2 * scale)
    rel = np.abs(g - ref).max() / scale
    assert rel < 1.6e-2, rel
    # no row of the output left unwritten (stale or NaN)
    assert np.isfinite(got.astype(np.float32)).all()


def test_plain_gemm_at_benchmark_shape(mx):
    """The same launch without the row factor (the matmul of the sweep's
    projections uses the plain epilogue)."""
    from phew_b200.workloads import normed_matmul_inputs

    x, w = normed_matmul_inputs("typical", 0)
    got = np.asarray(mx.array(x) @ mx.array(w))
    rows = _normed_rows(x.shape[0])
    ref = (x[rows].astype(np.float32) @ w.astype(np.float32)).astype(BF16).astype(np.float64)
    g = got[rows].astype(np.float64)
    scale = float(np.sqrt(np.mean(ref * ref)))
    np.testing.assert_allclose(g, ref, rtol=2e-2, atol=2e-2 * scale)
