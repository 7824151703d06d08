"""Runtime-compiled kernels: the ``mx.fast.cuda_kernel`` factory.

``CudaKernel`` is this backend's counterpart of the object that
``mx.fast.metal_kernel(name, input_names, output_names, source, header)``
returns (phew ``ir/importer.py:55-94``; emitted at ``emit/codegen.py:488-495``).
Calling it with ``inputs, output_shapes, output_dtypes, grid, threadgroup,
template`` (the call emitted at ``emit/codegen.py:584-592``) allocates the
outputs, wraps the body in an ``extern "C"`` signature built from the
argument dtypes, compiles it once with NVRTC for sm_100a (through the C ABI,
cached by source hash) and launches it on the current stream.

As in MLX, ``grid`` counts threads (not blocks) and ``threadgroup`` is the
block shape; blocks = ceil(grid / threadgroup) per axis.
"""

from __future__ import annotations

import ctypes
import hashlib
import math
import re
from typing import Any, Sequence

import torch

from . import _native
from . import dtypes as dt
from .emit.cuda_codegen import CTYPE, dtype_name

PRELUDE = r"""
// ---- phew_b200 kernel prelude ------------------------------------------
struct phew_f16 { unsigned short x; };
struct phew_bf16 { unsigned short x; };
typedef unsigned int phew_u32;
typedef unsigned long long phew_uptr;

__device__ __forceinline__ float phew_h2f(unsigned short h) {
  float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ unsigned short phew_f2h(float f) {
  unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
__device__ __forceinline__ float phew_bf2f(unsigned short b) {
  return __uint_as_float(((unsigned)b) << 16); }
__device__ __forceinline__ unsigned short phew_f2bf(float f) {
  unsigned short b; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(b) : "f"(f)); return b; }
// Row reductions and the softmax exponential of csrc/rows.cu (same order of
// operations, so fused softmax kernels give its bits).
__device__ __forceinline__ float phew_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float phew_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <bool IS_MAX>
__device__ __forceinline__ float phew_row_allreduce(float v, float* smem) {
  v = IS_MAX ? phew_warp_max(v) : phew_warp_sum(v);
  const int warps_per_row = blockDim.x / 32;
  if (warps_per_row == 1) return v;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* row_smem = smem + threadIdx.y * 32;
  __syncthreads();
  if (lane == 0) row_smem[warp] = v;
  __syncthreads();
  float r = lane < warps_per_row ? row_smem[lane] : (IS_MAX ? __int_as_float(0xff800000u) : 0.f);
  r = IS_MAX ? phew_warp_max(r) : phew_warp_sum(r);
  return r;
}
template <int ITEMSIZE>
__device__ __forceinline__ float phew_softmax_exp(float d) {
  if (ITEMSIZE == 4) return expf(d);
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d * 1.44269504088896341f));
  return y;
}
__device__ __forceinline__ float phew_rnd_f16(float f) { return phew_h2f(phew_f2h(f)); }
__device__ __forceinline__ float phew_rnd_bf16(float f) { return phew_bf2f(phew_f2bf(f)); }

__device__ __forceinline__ float phew_ld(phew_f16 v) { return phew_h2f(v.x); }
__device__ __forceinline__ float phew_ld(phew_bf16 v) { return phew_bf2f(v.x); }
__device__ __forceinline__ float phew_ld(float v) { return v; }
template <typename T> __device__ __forceinline__ T phew_ld(T v) { return v; }
__device__ __forceinline__ phew_f16 phew_st_f16(float v) { phew_f16 r; r.x = phew_f2h(v); return r; }
__device__ __forceinline__ phew_bf16 phew_st_bf16(float v) { phew_bf16 r; r.x = phew_f2bf(v); return r; }
__device__ __forceinline__ float phew_st_f32(float v) { return v; }
template <typename T> __device__ __forceinline__ T phew_st_raw(T v) { return v; }

// 16-byte vectors of V elements.
template <typename T, int V>
struct alignas((sizeof(T) * V) >= 16 ? 16 : (sizeof(T) * V)) phew_vec { T v[V]; };

template <typename T, int V>
__device__ __forceinline__ phew_vec<T, V> phew_ldv(const T* p) {
  phew_vec<T, V> r;
  constexpr int B = sizeof(T) * V;
  if constexpr (B % 16 == 0) {
#pragma unroll
    for (int i = 0; i < B / 16; ++i) {
      phew_u32* d = reinterpret_cast<phew_u32*>(&r) + 4 * i;
      asm("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
          : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
          : "l"(reinterpret_cast<const char*>(p) + 16 * i));
    }
  } else if constexpr (B == 8) {
    phew_u32* d = reinterpret_cast<phew_u32*>(&r);
    asm("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(d[0]), "=r"(d[1]) : "l"(p));
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = p[i];
  }
  return r;
}

// Asynchronous 16-byte global -> shared copies (cp.async): issue, close the
// group, wait until at most N groups are still in flight.
__device__ __forceinline__ void phew_cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
               :: "r"((unsigned)__cvta_generic_to_shared(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void phew_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void phew_cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void phew_cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// A vector from shared (or any generic) memory, 16-byte aligned.
template <typename T, int V>
__device__ __forceinline__ phew_vec<T, V> phew_ldv_s(const T* p) {
  return *reinterpret_cast<const phew_vec<T, V>*>(p);
}

template <typename T, int V>
__device__ __forceinline__ void phew_stv(T* p, const phew_vec<T, V>& r) {
  constexpr int B = sizeof(T) * V;
  if constexpr (B % 16 == 0) {
#pragma unroll
    for (int i = 0; i < B / 16; ++i) {
      const phew_u32* s = reinterpret_cast<const phew_u32*>(&r) + 4 * i;
      asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};"
                   :: "l"(reinterpret_cast<char*>(p) + 16 * i),
                      "r"(s[0]), "r"(s[1]), "r"(s[2]), "r"(s[3]) : "memory");
    }
  } else if constexpr (B == 8) {
    const phew_u32* s = reinterpret_cast<const phew_u32*>(&r);
    asm volatile("st.global.v2.u32 [%0], {%1, %2};" :: "l"(p), "r"(s[0]), "r"(s[1]) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = r.v[i];
  }
}

// Packed pairs of 16-bit floats.
template <typename T, int V>
__device__ __forceinline__ phew_u32 phew_pair(const phew_vec<T, V>& v, int p) {
  return reinterpret_cast<const phew_u32*>(&v)[p]; }
template <typename T, int V>
__device__ __forceinline__ void phew_set_pair(phew_vec<T, V>& v, int p, phew_u32 x) {
  reinterpret_cast<phew_u32*>(&v)[p] = x; }
__device__ __forceinline__ phew_u32 phew_splat2(phew_f16 s) { return (phew_u32)s.x | ((phew_u32)s.x << 16); }
__device__ __forceinline__ phew_u32 phew_splat2(phew_bf16 s) { return (phew_u32)s.x | ((phew_u32)s.x << 16); }

#define PHEW_PACKED_BINOP(NAME, INSTR) \
  __device__ __forceinline__ phew_u32 NAME(phew_u32 a, phew_u32 b) { \
    phew_u32 d; asm(INSTR " %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d; }
PHEW_PACKED_BINOP(phew_h2_add, "add.rn.f16x2")
PHEW_PACKED_BINOP(phew_h2_sub, "sub.rn.f16x2")
PHEW_PACKED_BINOP(phew_h2_mul, "mul.rn.f16x2")
PHEW_PACKED_BINOP(phew_b2_add, "add.rn.bf16x2")
PHEW_PACKED_BINOP(phew_b2_sub, "sub.rn.bf16x2")
PHEW_PACKED_BINOP(phew_b2_mul, "mul.rn.bf16x2")
#undef PHEW_PACKED_BINOP
__device__ __forceinline__ phew_u32 phew_h2_neg(phew_u32 a) { return a ^ 0x80008000u; }
__device__ __forceinline__ phew_u32 phew_h2_abs(phew_u32 a) { return a & 0x7fff7fffu; }
__device__ __forceinline__ phew_u32 phew_b2_neg(phew_u32 a) { return a ^ 0x80008000u; }
__device__ __forceinline__ phew_u32 phew_b2_abs(phew_u32 a) { return a & 0x7fff7fffu; }
__device__ __forceinline__ float phew_h2_lo(phew_u32 a) { return phew_h2f((unsigned short)(a & 0xffffu)); }
__device__ __forceinline__ float phew_h2_hi(phew_u32 a) { return phew_h2f((unsigned short)(a >> 16)); }
__device__ __forceinline__ float phew_b2_lo(phew_u32 a) { return __uint_as_float(a << 16); }
__device__ __forceinline__ float phew_b2_hi(phew_u32 a) { return __uint_as_float(a & 0xffff0000u); }
__device__ __forceinline__ phew_u32 phew_h2_pack(float lo, float hi) {
  phew_u32 d; asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo)); return d; }
__device__ __forceinline__ phew_u32 phew_b2_pack(float lo, float hi) {
  phew_u32 d; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo)); return d; }

// Transcendentals for nodes whose results are rounded to 16-bit floats:
// relative error about 2^-20, far below the 2^-11 / 2^-8 of the result.
__device__ __forceinline__ float phew_ex2(float x) {
  float y; asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float phew_rcp(float x) {
  float y; asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
// e^x = 2^(x log2 e)
__device__ __forceinline__ float phew_exp16(float x) { return phew_ex2(x * 1.4426950408889634f); }
// Precise forms (two transcendental-unit ops each):
// sigmoid(x) = 1 / (1 + e^-x)
__device__ __forceinline__ float phew_sigmoid16p(float x) { return phew_rcp(1.0f + phew_exp16(-x)); }
// tanh(x) = sign(x) (1 - 2 / (e^{2|x|} + 1)).  The subtraction loses bits as
// |x| shrinks (about 2^-14.5 relative at |x| = 2^-8); below 2^-8,
// tanh(x) = x to within x^3/3 < 2^-16 |x|, so x itself is returned.
__device__ __forceinline__ float phew_tanh16p(float x) {
  const float ax = fabsf(x);
  const float big = 1.0f - 2.0f * phew_rcp(phew_ex2(ax * 2.8853900817779268f) + 1.0f);
  return ax < 0.00390625f ? x : copysignf(big, x);
}
// Default forms (one transcendental-unit op each): the hardware tanh
// approximation (relative error about 2^-11, i.e. at most one or two ulps of
// the 16-bit result), and sigmoid(x) = (1 + tanh(x / 2)) / 2.
__device__ __forceinline__ float phew_tanh16(float x) {
  float y; asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float phew_sigmoid16(float x) {
  return fmaf(0.5f, phew_tanh16(0.5f * x), 0.5f); }

// numpy semantics for the ops below (NaN-propagating max/min, Python-style
// remainder and floor division).
__device__ __forceinline__ float phew_maximum(float a, float b) {
  return isnan(a) ? a : (isnan(b) ? b : (a > b ? a : b)); }
__device__ __forceinline__ float phew_minimum(float a, float b) {
  return isnan(a) ? a : (isnan(b) ? b : (a < b ? a : b)); }
__device__ __forceinline__ float phew_logaddexp(float a, float b) {
  const float m = fmaxf(a, b);
  if (isinf(m) && a == b) return m;
  return __fadd_rn(m, log1pf(expf(-fabsf(__fsub_rn(a, b))))); }
__device__ __forceinline__ float phew_sign(float a) {
  return a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : a); }
__device__ __forceinline__ float phew_remainder(float a, float b) {
  float r = fmodf(a, b);
  if (r != 0.0f && ((r < 0.0f) != (b < 0.0f))) r = __fadd_rn(r, b);
  return r; }
template <typename T> __device__ __forceinline__ T phew_floordiv_i(T a, T b) {
  if (b == 0) return 0;
  T q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) q -= 1;
  return q; }
template <typename T> __device__ __forceinline__ T phew_remainder_i(T a, T b) {
  if (b == 0) return 0;
  T r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) r += b;
  return r; }
// ---- end of prelude -----------------------------------------------------
"""

_NAME_RE = re.compile(r"^[A-Za-z_][A-Za-z0-9_]*$")


def _ctype_of(d) -> str:
    return CTYPE[dtype_name(d)]


def full_source(name: str, input_names, output_names, source: str, header: str,
                in_dtypes, out_dtypes, template=()) -> str:
    """The translation unit compiled for one (kernel, dtype signature)."""
    params = [
        f"const {_ctype_of(d)}* __restrict__ {n}" for n, d in zip(input_names, in_dtypes)
    ] + [f"{_ctype_of(d)}* __restrict__ {n}" for n, d in zip(output_names, out_dtypes)]
    # Element counts of every array follow the buffers (`<name>_size`).
    params += [f"const unsigned long long {n}_size" for n in list(input_names) + list(output_names)]
    tmpl_lines = []
    for k, v in template or ():
        if isinstance(v, bool):
            tmpl_lines.append(f"constexpr bool {k} = {'true' if v else 'false'};")
        elif isinstance(v, int):
            tmpl_lines.append(f"constexpr long long {k} = {v}LL;")
        else:
            tmpl_lines.append(f"typedef {_ctype_of(dt.from_any(v))} {k};")
    return (
        PRELUDE
        + (header or "")
        + "\n"
        + "\n".join(tmpl_lines)
        + f'\nextern "C" __global__ void {name}({", ".join(params)}) {{\n'
        + source
        + "\n}\n"
    )


class CudaKernel:
    """A runtime-compiled CUDA kernel with MLX ``metal_kernel`` call semantics."""

    def __init__(
        self,
        name: str,
        input_names: Sequence[str],
        output_names: Sequence[str],
        source: str,
        header: str = "",
        ensure_row_contiguous: bool = True,
        atomic_outputs: bool = False,
    ) -> None:
        safe = re.sub(r"[^A-Za-z0-9_]", "_", name) or "kernel"
        if not _NAME_RE.match(safe):
            safe = "k_" + safe
        self.name = safe
        self.input_names = list(input_names)
        self.output_names = list(output_names)
        self.source = source
        self.header = header
        self.ensure_row_contiguous = ensure_row_contiguous
        self.atomic_outputs = atomic_outputs
        self._handles: dict[tuple, int] = {}

    def _handle(self, in_dtypes, out_dtypes, template) -> int:
        key = (
            tuple(dtype_name(d) for d in in_dtypes),
            tuple(dtype_name(d) for d in out_dtypes),
            tuple((k, repr(v)) for k, v in (template or ())),
        )
        h = self._handles.get(key)
        if h is None:
            src = full_source(self.name, self.input_names, self.output_names, self.source,
                              self.header, in_dtypes, out_dtypes, template)
            out = ctypes.c_uint64(0)
            _native.call("phew_compile", src.encode(), self.name.encode(), ctypes.byref(out))
            h = out.value
            self._handles[key] = h
        return h

    def __call__(
        self,
        inputs: Sequence[Any],
        output_shapes: Sequence[Sequence[int]],
        output_dtypes: Sequence[Any],
        grid: Sequence[int],
        threadgroup: Sequence[int],
        template: Sequence[tuple[str, Any]] | None = None,
        init_value: float | None = None,
        verbose: bool = False,
        stream: Any = None,
    ):
        from .mx.core import array, asarray_device, empty

        if len(inputs) != len(self.input_names):
            raise ValueError(
                f"{self.name}: expected {len(self.input_names)} inputs, got {len(inputs)}"
            )
        if len(output_shapes) != len(self.output_names) or len(output_dtypes) != len(
            self.output_names
        ):
            raise ValueError(f"{self.name}: need one shape and dtype per output")
        ins = [asarray_device(x, contiguous=self.ensure_row_contiguous) for x in inputs]
        out_dts = [dt.from_any(d) for d in output_dtypes]
        outs = [empty(tuple(int(s) for s in shp), d) for shp, d in zip(output_shapes, out_dts)]
        if init_value is not None:
            for o in outs:
                o._t.fill_(init_value)
        handle = self._handle([x.dtype for x in ins], out_dts, template)
        if verbose:
            print(full_source(self.name, self.input_names, self.output_names, self.source,
                              self.header, [x.dtype for x in ins], out_dts, template))
        g = tuple(int(v) for v in (tuple(grid) + (1, 1, 1))[:3])
        tg = tuple(int(v) for v in (tuple(threadgroup) + (1, 1, 1))[:3])
        if any(v <= 0 for v in tg):
            raise ValueError(f"{self.name}: threadgroup must be positive, got {tg}")
        blocks = tuple(max(1, math.ceil(a / b)) for a, b in zip(g, tg))
        if all(o.size == 0 for o in outs) or any(v == 0 for v in g):
            return outs
        check_io_contract(self.source, [x.shape for x in ins], [o.shape for o in outs], self.name)
        vals = [ctypes.c_void_p(x._t.data_ptr()) for x in ins + outs]
        vals += [ctypes.c_uint64(x.size) for x in ins + outs]
        argv = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.byref(p), ctypes.c_void_p) for p in vals])
        ptrs = vals
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        _native.call(
            "phew_launch", ctypes.c_uint64(handle), argv, len(ptrs), *blocks, *tg, 0,
            ctypes.c_void_p(st),
        )
        return outs


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def check_io_contract(source: str, in_shapes, out_shapes, name: str = "kernel") -> None:
    """Refuse a launch that would index outside its arrays.

    Bodies emitted by ``SubgraphCUDACodegen`` carry a ``// phew-io:`` line
    describing how each input is indexed from the flat output index; this
    checks the runtime shapes against it (bodies without the line are the
    caller's responsibility, as with MLX's custom kernels).
    """
    from .emit.cuda_codegen import IO_TAG

    pos = source.find(IO_TAG)
    if pos < 0:
        return
    line = source[pos + len(IO_TAG):].split("\n", 1)[0].split()
    n = _numel(out_shapes[0]) if out_shapes else 0
    for o in out_shapes:
        if _numel(o) != n:
            raise ValueError(f"{name}: fused outputs must all have {n} elements, got {o}")
    # A fused row reduction writes one value per row of `rowred` elements:
    # its inputs are indexed over rows x rowred.
    for tok in line:
        if tok.startswith("rowred="):
            n *= int(tok[len("rowred="):])
            if any(t.startswith("inp") and "=general" in t for t in line):
                raise ValueError(f"{name}: general broadcasts are not fused into reductions")
        # A row map reduces and rewrites rows of exactly `rowlen` elements.
        if tok.startswith("rowlen="):
            k = int(tok[len("rowlen="):])
            if not out_shapes or not out_shapes[0] or int(out_shapes[0][-1]) != k:
                raise ValueError(f"{name}: the kernel maps rows of {k} elements, output {out_shapes}")
        # A kernel whose row order is baked in serves exactly `rows` rows.
        if tok.startswith("rows="):
            k = int(tok[len("rows="):])
            if not out_shapes or not out_shapes[0] or _numel(out_shapes[0]) != k * int(out_shapes[0][-1]):
                raise ValueError(f"{name}: the kernel's row order covers {k} rows, output {out_shapes}")
    for tok in line:
        if tok == "idx32" and n >= 2**31 - 2**20:
            raise ValueError(f"{name}: {n} elements overflow the kernel's 32-bit indexing")
        if tok.startswith("out="):
            continue
        if not tok.startswith("inp"):
            continue
        key, spec = tok.split("=", 1)
        k = int(key[3:])
        m = _numel(in_shapes[k])
        cls, _, arg = spec.partition(":")
        ok = True
        if cls == "full":
            ok = m == n
        elif cls == "scalar":
            ok = m == 1
        elif cls == "suffix":
            ext = int(arg)
            ok = m == ext and n % ext == 0
        elif cls == "prefix":
            ext = int(arg)
            ok = m * ext == n
        elif cls == "general":
            baked_out = [t for t in line if t.startswith("out=")][0][4:]
            ok = (arg == "x".join(str(int(s)) for s in in_shapes[k])
                  and baked_out == "x".join(str(int(s)) for s in out_shapes[0]))
        if not ok:
            raise ValueError(
                f"{name}: input {k} of shape {tuple(in_shapes[k])} does not fit the kernel's "
                f"'{spec}' indexing for {n} output elements"
            )


def source_digest(source: str) -> str:
    return hashlib.sha1(source.encode()).hexdigest()[:12]
