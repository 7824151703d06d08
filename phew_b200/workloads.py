"""Benchmark workloads: harness functions, seeded inputs and fused chains.

Each workload is a phew harness in the shape of the reference's examples
(``examples/rms_norm.py:11-32``: a function ``fn`` written against ``mx``
plus ``input_factory(size_label, seed) -> (args, kwargs)``).  Functions are
built for a given ``mx`` namespace (``phew_b200.mx`` on the GPU, the oracle
on the CPU), so the same definition runs on both.

Inputs are drawn on the host with ``np.random.default_rng(seed)`` as the
reference examples do (``examples/rms_norm.py:27-31``); public datasets are
not involved.  Shapes follow the benchmark definitions:

* rms_norm       x float32 (n, 2048), n = 256 / 1024 / 4096, w = ones(2048)
* gelu_chain     z = tanh-GELU(x*a + b) * sigmoid(c) + x, x, c float16
                 (rows, 8192) N(0,1), a, b float16 (8192,) U(-1,1),
                 rows = 1024 / 4096 / 8192 (4096 is the benchmark shape)
* attention      softmax(q @ k^T * s + mask) @ v, bf16 (4, 32, L, 128),
                 L = 512 / 2048 / 4096, s = 1/sqrt(128), causal additive mask
* normed_matmul  (x @ W) * rsqrt(mean(x*x, -1) + 1e-5), x bf16 (M, 4096)
                 N(0,1), W bf16 (4096, 4096) N(0, 1/4096), M = 2048/8192/16384
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable

import ml_dtypes
import numpy as np

from .graph import NodeSpec, const, ew, inp

BF16 = np.dtype(ml_dtypes.bfloat16)


@dataclass
class Workload:
    name: str
    make_fn: Callable[[Any], Callable]
    host_inputs: Callable[[str, int], list]
    sizes: dict
    dtype: str

    def input_factory(self, mx) -> Callable[[str, int], tuple[list, dict]]:
        def factory(size_label: str, seed: int):
            return [mx.array(a) for a in self.host_inputs(size_label, seed)], {}

        return factory


# ---------------------------------------------------------------------------
# rms_norm (fp32)
# ---------------------------------------------------------------------------

RMS_ROWS = {"small": 256, "typical": 1024, "large": 4096}
RMS_COLS = 2048


def rms_norm_fn(mx):
    def fn(x, w):
        return x * mx.rsqrt(mx.mean(x * x, axis=-1, keepdims=True) + 1e-5) * w

    return fn


def layer_norm_fn(mx):
    """A layer norm written out with mean / var, the shape the reference's
    primitive substitution rewrites to ``mx.fast.layer_norm``
    (``rules/primitive_subst.py:246-333``)."""
    def fn(x, w, b):
        mu = mx.mean(x, axis=-1, keepdims=True)
        var = mx.var(x, axis=-1, keepdims=True)
        return (x - mu) / mx.sqrt(var + 1e-5) * w + b

    return fn


def rope_fn(mx, half: int = 64):
    """Rotary embedding written out with cos / sin of a position-angle table
    and a concatenation of the rotated halves, the shape the reference's
    substitution rewrites to ``mx.fast.rope`` (``rules/primitive_subst.py:339-407``;
    the rewrite keeps only x and uses the default base and positions)."""
    def fn(x, angles):
        c, s = mx.cos(angles), mx.sin(angles)
        x1, x2 = x[..., :half], x[..., half:]
        return mx.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1)

    return fn


def rms_norm_inputs(size: str, seed: int, rows: int | None = None):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows or RMS_ROWS[size], RMS_COLS)).astype(np.float32)
    w = np.ones((RMS_COLS,), np.float32)
    return [x, w]


# ---------------------------------------------------------------------------
# elementwise chain (fp16)
# ---------------------------------------------------------------------------

CHAIN_ROWS = {"small": 1024, "typical": 4096, "large": 8192}
CHAIN_COLS = 8192
SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def gelu_chain_fn(mx):
    def fn(x, a, b, c):
        y = x * a + b
        g = (y * 0.5) * (mx.tanh((y + y * y * y * 0.044715) * SQRT_2_OVER_PI) + 1.0)
        return g * mx.sigmoid(c) + x

    return fn


def gelu_chain_inputs(size: str, seed: int, rows: int | None = None):
    rng = np.random.default_rng(seed)
    r = rows if rows is not None else CHAIN_ROWS[size]
    x = rng.standard_normal((r, CHAIN_COLS), dtype=np.float32).astype(np.float16)
    a = rng.uniform(-1.0, 1.0, (CHAIN_COLS,)).astype(np.float16)
    b = rng.uniform(-1.0, 1.0, (CHAIN_COLS,)).astype(np.float16)
    c = rng.standard_normal((r, CHAIN_COLS), dtype=np.float32).astype(np.float16)
    return [x, a, b, c]


def gelu_chain_nodes(rows: int, cols: int = CHAIN_COLS, dtype: str = "float16"):
    """The fused chain of ``gelu_chain_fn`` as the fusion pass finds it:
    (chain nodes in topological order, external inputs, external outputs).

    Node order and Constant placement match what phew's tracer records for
    the harness function (one Constant per Python scalar, recorded just
    before its use, ``ir/importer.py:171-186``).
    """
    S = (rows, cols)
    x, a, b, c = inp(S, dtype, "x"), inp((cols,), dtype, "a"), inp((cols,), dtype, "b"), inp(S, dtype, "c")
    n_xa = ew("mul", x, a)
    y = ew("add", n_xa, b)
    k_half = const(0.5, dtype)
    y_half = ew("mul", y, k_half)
    yy = ew("mul", y, y)
    yyy = ew("mul", yy, y)
    k_c = const(0.044715, dtype)
    cub = ew("mul", yyy, k_c)
    inner = ew("add", y, cub)
    k_s = const(SQRT_2_OVER_PI, dtype)
    arg = ew("mul", inner, k_s)
    t = ew("tanh", arg)
    k_one = const(1.0, dtype)
    t1 = ew("add", t, k_one)
    g = ew("mul", y_half, t1)
    s = ew("sigmoid", c)
    gs = ew("mul", g, s)
    z = ew("add", gs, x)
    chain = [n_xa, y, k_half, y_half, yy, yyy, k_c, cub, inner, k_s, arg, t, k_one, t1, g, s, gs, z]
    return chain, [x, a, b, c], [z]


def gelu_chain_bytes(rows: int, cols: int = CHAIN_COLS) -> int:
    """Algorithmic HBM bytes of one fused launch: read x, c, a, b; write z."""
    return 3 * rows * cols * 2 + 2 * cols * 2


# ---------------------------------------------------------------------------
# attention (bf16, causal)
# ---------------------------------------------------------------------------

ATTN_B, ATTN_H, ATTN_D = 4, 32, 128
ATTN_L = {"small": 512, "typical": 2048, "large": 4096}


def attention_fn(mx):
    scale = 1.0 / math.sqrt(ATTN_D)

    def fn(q, k, v, mask):
        s = (q @ k.transpose(0, 1, 3, 2)) * scale + mask
        return mx.softmax(s, axis=-1) @ v

    return fn


def causal_mask(L: int) -> np.ndarray:
    m = np.zeros((L, L), np.float32)
    m[np.triu_indices(L, 1)] = -np.inf
    return m.astype(BF16)


def attention_inputs(size: str, seed: int, L: int | None = None, B: int = ATTN_B, H: int = ATTN_H):
    rng = np.random.default_rng(seed)
    L = L or ATTN_L[size]
    shp = (B, H, L, ATTN_D)
    q = rng.standard_normal(shp, dtype=np.float32).astype(BF16)
    k = rng.standard_normal(shp, dtype=np.float32).astype(BF16)
    v = rng.standard_normal(shp, dtype=np.float32).astype(BF16)
    return [q, k, v, causal_mask(L)]


def attention_flops(B: int, H: int, L: int, D: int, causal: bool = True) -> int:
    full = 4 * B * H * L * L * D
    return full // 2 if causal else full


# ---------------------------------------------------------------------------
# normed matmul (bf16)
# ---------------------------------------------------------------------------

NMM_K = NMM_N = 4096
NMM_M = {"small": 2048, "typical": 8192, "large": 16384}


def normed_matmul_fn(mx):
    def fn(x, W):
        return (x @ W) * mx.rsqrt(mx.mean(x * x, axis=-1, keepdims=True) + 1e-5)

    return fn


def normed_matmul_inputs(size: str, seed: int, M: int | None = None):
    rng = np.random.default_rng(seed)
    M = M or NMM_M[size]
    x = rng.standard_normal((M, NMM_K), dtype=np.float32).astype(BF16)
    W = (rng.standard_normal((NMM_K, NMM_N), dtype=np.float32) / np.float32(64.0)).astype(BF16)
    return [x, W]


# ---------------------------------------------------------------------------
# decoder block (bf16): the verification-sweep workload
# ---------------------------------------------------------------------------

DECODER_SEQ = {"small": 512, "typical": 2048, "large": 8192}


@dataclass(frozen=True)
class DecoderDims:
    batch: int = 8
    dim: int = 4096
    heads: int = 32
    hidden: int = 14336

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


DECODER_FULL = DecoderDims()
DECODER_TINY = DecoderDims(batch=2, dim=256, heads=2, hidden=512)
DECODER_TINY_SEQ = {"small": 128, "typical": 256, "large": 384}


def decoder_block_fn(mx, dims: DecoderDims = DECODER_FULL):
    """Pre-norm decoder block: RMSNorm -> fused QKV projection -> causal
    attention (additive mask input) -> output projection + residual ->
    SwiGLU MLP whose norm is applied after the gate/up projections (the
    normed-matmul form (h @ W) * rsqrt(mean(h*h) + eps)) -> residual."""
    H, D, C = dims.heads, dims.head_dim, dims.dim
    scale = 1.0 / math.sqrt(D)

    def fn(x, w_norm, w_qkv, w_o, w_gate, w_up, w_down, mask):
        B, T = x.shape[0], x.shape[1]
        h = x * mx.rsqrt(mx.mean(x * x, axis=-1, keepdims=True) + 1e-5) * w_norm
        qkv = (h @ w_qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        s = (q @ k.transpose(0, 1, 3, 2)) * scale + mask
        a = (mx.softmax(s, axis=-1) @ v).transpose(0, 2, 1, 3).reshape(B, T, C)
        h1 = x + a @ w_o
        r = mx.rsqrt(mx.mean(h1 * h1, axis=-1, keepdims=True) + 1e-5)
        g = (h1 @ w_gate) * r
        u = (h1 @ w_up) * r
        return h1 + ((g * mx.sigmoid(g)) * u) @ w_down

    return fn


def decoder_arg_shapes(seq: int, dims: DecoderDims = DECODER_FULL) -> list[tuple]:
    C, F = dims.dim, dims.hidden
    return [(dims.batch, seq, C), (C,), (C, 3 * C), (C, C), (C, F), (C, F), (F, C), (seq, seq)]


def decoder_fan_in(dims: DecoderDims = DECODER_FULL) -> list[int]:
    C, F = dims.dim, dims.hidden
    return [1, 1, C, C, C, C, F, 1]


def decoder_inputs(size: str, seed: int, dims: DecoderDims = DECODER_FULL, seqs=None):
    """Host inputs (numpy, bf16): x ~ N(0,1), weights ~ N(0, 1/fan_in), norm
    weight = ones, causal additive mask."""
    seq = (seqs or DECODER_SEQ)[size]
    rng = np.random.default_rng(seed)
    out = []
    for i, (shp, fan) in enumerate(zip(decoder_arg_shapes(seq, dims), decoder_fan_in(dims))):
        if i == 1:
            out.append(np.ones(shp, np.float32).astype(BF16))
        elif i == 7:
            out.append(causal_mask(seq))
        else:
            a = rng.standard_normal(shp, dtype=np.float32)
            if fan > 1:
                a *= np.float32(1.0 / math.sqrt(fan))
            out.append(a.astype(BF16))
    return out


def decoder_flops(seq: int, dims: DecoderDims = DECODER_FULL) -> int:
    T = dims.batch * seq
    C, F = dims.dim, dims.hidden
    proj = 2 * T * (C * 3 * C + C * C + 2 * C * F + F * C)
    attn = 2 * 2 * dims.batch * dims.heads * seq * seq * dims.head_dim
    return proj + attn


WORKLOADS = {
    "rms_norm": Workload("rms_norm", rms_norm_fn, rms_norm_inputs, RMS_ROWS, "float32"),
    "gelu_chain": Workload("gelu_chain", gelu_chain_fn, gelu_chain_inputs, CHAIN_ROWS, "float16"),
    "attention": Workload("attention", attention_fn, attention_inputs, ATTN_L, "bfloat16"),
    "normed_matmul": Workload("normed_matmul", normed_matmul_fn, normed_matmul_inputs, NMM_M, "bfloat16"),
}

_ = NodeSpec  # re-exported builders live in phew_b200.graph
