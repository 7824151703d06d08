/*
 * phew_b200.h — C ABI of the B200 execution backend for phew's
 * candidate-evaluation path.
 *
 * The reference reaches its device through MLX: `mx.fast.metal_kernel`
 * objects built from generated MSL, the `mx.fast.*` primitives that the
 * primitive-substitution pass emits, `a @ b`, `mx.softmax`, and the
 * numpy comparison loop of its equivalence checker.  Each entry point below
 * replaces one of those call sites; the comment on each names the reference
 * file:line it stands in for (paths relative to the phew project root).
 *
 * Conventions
 *   - Every function returns an int status: PHEW_OK (0) or a PHEW_ERR_* code.
 *     phew_last_error() returns the message of the last failure on the
 *     calling thread.
 *   - Pointers named x/y/q/k/v/... are DEVICE pointers of the current CUDA
 *     device (in practice `torch.Tensor.data_ptr()`).  The library never
 *     frees memory it did not allocate.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  All work is asynchronous on that stream.
 *   - dtype codes: PHEW_F32, PHEW_F16, PHEW_BF16 (phew.ir.dtype.Dtype
 *     float32 / float16 / bfloat16, ir/dtype.py:6-9).
 *   - Shapes are row-major and contiguous unless strides are given.
 */
#ifndef PHEW_B200_H
#define PHEW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PHEW_OK 0
#define PHEW_ERR_INVALID 1     /* bad argument (null pointer, bad shape, bad dtype) */
#define PHEW_ERR_CUDA 2        /* a CUDA runtime call failed */
#define PHEW_ERR_COMPILE 3     /* NVRTC compilation failed; log in phew_last_error */
#define PHEW_ERR_UNSUPPORTED 4 /* valid request this build does not implement */
#define PHEW_ERR_TIMEOUT 5     /* a bounded device-side wait gave up */
#define PHEW_ERR_NOT_FOUND 6   /* unknown kernel handle or symbol */

/* ---- dtype codes ------------------------------------------------------- */
#define PHEW_F32 0
#define PHEW_F16 1
#define PHEW_BF16 2

/* ---- reduction op codes (phew.ir.ops.Reduce.op, ir/ops.py:43-52) -------- */
#define PHEW_REDUCE_SUM 0
#define PHEW_REDUCE_MEAN 1
#define PHEW_REDUCE_MAX 2
#define PHEW_REDUCE_MIN 3
#define PHEW_REDUCE_PROD 4

/* ---- library / device -------------------------------------------------- */

/* ABI version of this library (bumped on any signature change). */
int phew_abi_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len).  Returns the length of the full message. */
int phew_last_error(char* buf, size_t len);

/* Selects `device` for the calling thread and caches its properties.
 * Replaces the implicit MLX device setup behind `mx.metal.is_available()` /
 * `mx.device_info()` (optimizer.py:114-116). */
int phew_init(int device);

typedef struct phew_device_info {
  int sm_count;
  int cc_major;
  int cc_minor;
  int max_smem_per_block_optin;
  int64_t l2_bytes;
  int64_t hbm_bytes;
  char name[128];
} phew_device_info;

int phew_device_query(int device, phew_device_info* out);

/* ---- runtime-compiled kernels (NVRTC, sm_100a) ------------------------- */

/* Compiles CUDA C++ `source` with NVRTC for sm_100a and loads kernel
 * `kernel_name` (an extern "C" __global__ symbol of the source).  Results are
 * cached by a hash of (source, kernel_name); *handle identifies the kernel.
 * On PHEW_ERR_COMPILE the NVRTC log is available from phew_last_error().
 * Replaces `mx.fast.metal_kernel(name, input_names, output_names, source,
 * header)` kernel construction (ir/importer.py:55-94, emit/codegen.py:488-495),
 * whose MSL MLX JIT-compiles on first call. */
int phew_compile(const char* source, const char* kernel_name, uint64_t* handle);

/* Launches a compiled kernel.  `args` holds `nargs` pointers to the argument
 * values (cudaLaunchKernel convention).  grid/block are in blocks/threads.
 * Replaces the call of a metal_kernel object (emit/codegen.py:584-592). */
int phew_launch(uint64_t handle, void** args, int nargs,
                unsigned grid_x, unsigned grid_y, unsigned grid_z,
                unsigned block_x, unsigned block_y, unsigned block_z,
                size_t dynamic_smem, void* stream);

/* Number of kernels this library has launched in this process (its own
 * kernels and phew_launch'ed ones; launches recorded into a CUDA graph count
 * once, when captured).  A harness reads it around a timed region. */
int phew_launch_count(uint64_t* out);

/* Number of kernels currently held in the compile cache. */
int phew_compile_cache_size(void);

/* Copies the NVRTC log of the last compilation phew_compile ran on the
 * calling thread (warnings included; a cache hit runs none and leaves it)
 * into buf, NUL-terminated and truncated to len.  Returns the full length.
 * The log MLX prints when a metal_kernel source fails to build
 * (ir/importer.py:55-94 constructs the kernel; the error surfaces at
 * optimizer.py:293-297). */
int phew_compile_log(char* buf, size_t len);

/* ---- streams and timing ------------------------------------------------- */

/* A non-blocking CUDA stream (returned as void*), and its release.  The
 * reference runs everything on MLX's default stream; a binding that does
 * not own streams of its own gets them here. */
int phew_stream_create(void** stream);
int phew_stream_destroy(void* stream);

/* CUDA events for device-side timing: record on a stream, then the elapsed
 * milliseconds between two recorded events (waits for `stop`).  Replaces the
 * perf_counter pair around mx.eval / mx.synchronize in the reference's
 * benchmark loop (bench/harness.py:44-55). */
int phew_event_create(void** event);
int phew_event_record(void* event, void* stream);
int phew_event_elapsed_ms(void* start, void* stop, float* ms);
int phew_event_destroy(void* event);

/* Test hook for the failure path of the tensor-core pipelines, not for
 * production use.  The NEXT phew_gemm or phew_sdpa call on the calling
 * thread that launches a tcgen05 kernel leaves one of its producer's tile
 * loads unissued -- GEMM: ring position `stage` (the stage-th k-block load
 * of each CTA); attention: the V tile of key tile `stage` -- and bounds
 * each of its pipeline waits by `wait_limit_ns` (0 < limit <= 1 s) instead
 * of 1 s.  The consumers' waits then run out: the kernel sets the caller's
 * error flag to PHEW_ERR_TIMEOUT, lets the loads and MMAs it did issue land,
 * frees its TMEM and returns, and the device stays usable.  One-shot: the
 * call that uses it clears it.  No counterpart in the reference (MLX's
 * kernels have no bounded waits to exercise). */
int phew_test_inject_stall(int stage, uint64_t wait_limit_ns);

/* ---- hand-written primitives ------------------------------------------- */

/* y[r, :] = w * cast(x[r, :] * rsqrt(mean(x[r, :]^2) + eps)); w may be NULL
 * (no weight).  Sum of squares in fp32.  x, w, y share `dtype`.
 * Replaces `mx.fast.rms_norm(x, w, eps)` (emit/codegen.py:401-404, node
 * FastRMSNorm ir/ops.py:156-161 from rules/primitive_subst.py:63-145). */
int phew_rms_norm(const void* x, const void* w, void* y, int64_t rows,
                  int64_t cols, float eps, int dtype, void* stream);

/* y[r, :] = T(w * T((x[r, :] - mean) * rsqrt(var + eps)) + b) with the mean
 * and the biased variance of the row in fp32; w and b may each be NULL.
 * x, w, b, y share `dtype`.
 * Replaces `mx.fast.layer_norm(x, w, b, eps=)` (emit/codegen.py:406-411, node
 * FastLayerNorm ir/ops.py:165-168 from rules/primitive_subst.py:246-333). */
int phew_layer_norm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                    int64_t cols, float eps, int dtype, void* stream);

/* Rotary embedding of x viewed as [rows, D], rows = leading dims x L, row r
 * at position offset + r % L.  The first `dims` (even) features rotate in
 * pairs (i, i + dims/2), or (2i, 2i + 1) when traditional, by the angle
 * position * scale * base^(-2i/dims); the rest are copied.
 * Replaces `mx.fast.rope(x, dims, traditional=, base=, scale=, offset=)`
 * (emit/codegen.py:413-419, node FastRoPE ir/ops.py:172-179 from
 * rules/primitive_subst.py:339-407). */
int phew_rope(const void* x, void* y, int64_t rows, int64_t D, int64_t L, int dims,
              int traditional, float base, float scale, int64_t offset, int dtype,
              void* stream);

/* Row softmax over the last axis, fp32 internally, result in `dtype`.
 * Replaces `mx.softmax(x, axis=-1)` (emit/codegen.py:147-150; Reduce op
 * "softmax" recorded at ir/importer.py:494-506). */
int phew_softmax(const void* x, void* y, int64_t rows, int64_t cols,
                 int dtype, void* stream);

/* Reduction of x viewed as [outer, red, inner] over the middle axis into
 * y[outer, inner].  fp32 accumulation; y has the dtype of x.
 * Replaces mx.sum/mean/max/min/prod (emit/codegen.py:94-146). */
int phew_reduce(int op, const void* x, void* y, int64_t outer, int64_t red,
                int64_t inner, int dtype, void* stream);

/* Variance over the middle axis of x viewed as [outer, red, inner]:
 * fp32 mean, fp32 sum of squared deviations / (red - ddof), rounded once to
 * `dtype`.  Replaces mx.var (emit/codegen.py:94-146, Reduce op "var"). */
int phew_reduce_var(const void* x, void* y, int64_t outer, int64_t red, int64_t inner,
                    int ddof, int dtype, void* stream);

/* dst (contiguous) = src viewed with `shape` and element `src_strides`
 * (ndim <= 8).  Materialises Transpose / non-contiguous views
 * (emit/codegen.py:312-317 `mx.transpose`). */
int phew_copy_strided(const void* src, void* dst, int ndim,
                      const int64_t* shape, const int64_t* src_strides,
                      int elem_bytes, void* stream);

/* Strided-to-strided copy: element (i0..in) of `shape` moves from
 * src + sum(ik * src_strides[k]) to dst + sum(ik * dst_strides[k]) (element
 * units; dst_strides NULL = contiguous).  Writes into views of a larger
 * array: concatenate / stack / pad / slice_update / roll (codegen.py:94-476
 * array-manipulation ops). */
int phew_copy_strided_to(const void* src, void* dst, int ndim, const int64_t* shape,
                         const int64_t* src_strides, const int64_t* dst_strides,
                         int elem_bytes, void* stream);

/* Writes `bytes` bytes of `buf` so that the L2 holds none of the caller's
 * data afterwards (buf must be larger than the L2).  Used between timed
 * iterations; replaces nothing in the reference (bench/harness.py:28-90
 * times warm caches). */
int phew_l2_flush(void* buf, size_t bytes, void* stream);

/* ---- tensor-core GEMM -------------------------------------------------- */

/* C[b] = A[b] @ B[b] (+ optional fused row scale), fp32 accumulation on the
 * tcgen05 tensor cores with TMA-fed, 128B-swizzled shared-memory tiles.
 *   A: [M, K] rows of stride lda (elements), K contiguous.
 *   B: b_layout 0 -> [K, N] rows of stride ldb, N contiguous
 *      b_layout 1 -> [N, K] rows of stride ldb, K contiguous (e.g. k.T)
 *   C: [M, N] rows of stride ldc, dtype out_dtype.
 *   stride_a / stride_b / stride_c: element strides between batches; 0 on an
 *   operand broadcasts it over the batch.
 *   row_scale = 1 multiplies row m of the product by
 *   rsqrt(mean_k(A[m, k]^2) + eps) (the normed matmul
 *   (x @ W) * rsqrt(mean(x^2) + eps)): one pass over A computes the factor per
 *   row into stream-ordered memory (cudaMallocFromPoolAsync / cudaFreeAsync
 *   on `stream`, from a pool the library keeps per device, so graph capture
 *   records it), and the GEMM, launched as that pass's programmatic
 *   dependent, applies it to the fp32 accumulator in its epilogue.
 *   row_scale = 2 writes each row's sum of squares of A instead of the
 *   product (a diagnostic of the row statistic).
 *   error_flag (device int, may be NULL) receives PHEW_ERR_TIMEOUT if a
 *   bounded pipeline wait ran out.
 * in_dtype bf16/f16 use the tensor cores when every row stride and base is
 * 16-byte aligned; f32 and unaligned layouts use a SIMT kernel.
 * Replaces `a @ b` (emit/codegen.py:129-133) and the normed-matmul rewrite
 * rms_norm(x) @ W (rules/primitive_subst.py:156-240). */
int phew_gemm(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
              int64_t batch, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a,
              int64_t stride_b, int64_t stride_c, int b_layout, int in_dtype, int out_dtype,
              int row_scale, float eps, int* error_flag, void* stream);

/* phew_gemm over two batch axes with strides of their own: batch entry
 * (o, i), o < batch_outer, i < batch_inner, reads A at
 * o * stride_a_outer + i * stride_a_inner (elements) and B likewise, and
 * writes C at (o * batch_inner + i) * stride_c.  The attention operands that
 * an unfused candidate slices out of a fused qkv projection,
 * qkv.reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4), are such views (the
 * batch stride of q over heads is D, over the batch T * 3 * H * D): the GEMM
 * reads them in place (4-D TMA maps) instead of after a copy.  An operand is
 * batched over both axes (both strides non-zero) or over neither (both 0).
 * No row scale.  Replaces the same `a @ b` call sites as phew_gemm. */
int phew_gemm_batched2(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                       int64_t batch_outer, int64_t batch_inner, int64_t lda, int64_t ldb,
                       int64_t ldc, int64_t stride_a_outer, int64_t stride_a_inner,
                       int64_t stride_b_outer, int64_t stride_b_inner, int64_t stride_c,
                       int b_layout, int in_dtype, int out_dtype, int* error_flag, void* stream);

/* ---- attention --------------------------------------------------------- */

/* 1 when phew_sdpa's tensor-core kernel handles this shape/dtype
 * (D == 128, L % 128 == 0, bf16/f16). */
int phew_sdpa_supported(int64_t L, int64_t D, int dtype);

/* o = softmax(q k^T * scale (+ causal mask)) v for batch_heads independent
 * [L, D] slices stored contiguously ([B*H, L, D], D contiguous).  S = QK^T and
 * O += PV run on tcgen05 with TMEM accumulators; the softmax (running max with
 * lazy rescaling, exp2) runs between them on the CUDA cores; scores never
 * reach HBM.  causal = 1 masks key j > query i.  scale must be positive
 * (PHEW_ERR_INVALID otherwise).  error_flag as in phew_gemm.
 * Replaces mx.fast.scaled_dot_product_attention(q, k, v, scale=)
 * (emit/codegen.py:421-426; FastScaledDotProductAttention ir/ops.py:182-187,
 * produced by rules/primitive_subst.py:413-499). */
int phew_sdpa(const void* q, const void* k, const void* v, void* o, int64_t batch_heads,
              int64_t L, int64_t D, float scale, int causal, int dtype, int* error_flag,
              void* stream);

/* phew_sdpa on [batch][heads][L][D] views with strides of their own (row,
 * head, batch; elements, positive multiples of 8): q, k and v sliced out of
 * a fused qkv projection, qkv.reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4),
 * are read in place.  o is contiguous [batch * heads, L, D].  Replaces
 * the same call site as phew_sdpa. */
int phew_sdpa_strided(const void* q, const void* k, const void* v, void* o, int64_t batch,
                      int64_t heads, int64_t L, int64_t D, const int64_t* q_strides,
                      const int64_t* k_strides, const int64_t* v_strides, float scale, int causal,
                      int dtype, int* error_flag, void* stream);

/* ---- group-wise quantised weights --------------------------------------- */

/* out[r, c] = T(scales[r, c / g] * q[r, c] + biases[r, c / g]) for codes q
 * packed 32 / bits per uint32 along c (code j of a word in bits
 * [j*bits, (j+1)*bits)), scales / biases [rows, cols / g] in `dtype`.
 * The weight side of mx.quantized_matmul and of
 * mx.fast.quantized_scaled_dot_product_attention (emit/codegen.py:428-449;
 * QuantizedMatMul ir/ops.py:209-218 from rules/quantization.py:37-71). */
int phew_dequantize(const void* wq, const void* scales, const void* biases, void* out,
                    int64_t rows, int64_t cols, int group_size, int bits, int dtype,
                    void* stream);

/* The producer of that layout (mx.quantize, which the quantisation rewrite
 * assumes for the weights it packs, rules/quantization.py:37-71): per group
 * of g values along a row, scale = T(max((max - min) / (2^bits - 1), 1e-8)),
 * bias = T(min), q = clamp(rint((w - bias) / scale), 0, 2^bits - 1) in fp32
 * with IEEE division.  w [rows, cols] in `dtype`; wq [rows, cols * bits / 32]
 * uint32; scales / biases [rows, cols / g] in `dtype`. */
int phew_quantize(const void* w, void* wq, void* scales, void* biases, int64_t rows,
                  int64_t cols, int group_size, int bits, int dtype, void* stream);

/* ---- seeded inputs for the verification sweep -------------------------- */

#define PHEW_FILL_NORMAL 0       /* N(0, 1) * scale (Box-Muller)           */
#define PHEW_FILL_UNIFORM 1      /* U(-1, 1) * scale                       */
#define PHEW_FILL_ONE_HOT_ROWS 2 /* one `scale` per row of `cols`, at a seeded column */
#define PHEW_FILL_CONSTANT 3     /* every element = scale                  */

/* Fills n elements of `dtype` at `out` from a counter-based generator:
 * element i depends only on (seed, stream_id, i), so inputs are identical on
 * any GPU and for any number of GPUs.  Stands in for the host-side draws of
 * the reference's input factories and edge variants
 * (verify/checker.py:235-263) at sweep scale. */
int phew_fill(void* out, int64_t n, int64_t cols, int dtype, int kind, uint64_t seed,
              uint64_t stream_id, float scale, void* stream);

/* The same generator on `threads` host threads (<= 0: one per hardware
 * thread) into HOST memory `out` (pinned or pageable); synchronous.  The
 * reference's input factories draw on the host
 * (examples/rms_norm.py:27-31, verify/checker.py:246-263); a caller whose
 * inputs must start in host memory (an end-to-end sweep that copies them
 * in) draws here.  Normals are computed in SIMD loops (series forms of ln
 * and cos / sin, within 2.6e-7 relative of the exact transform), so they
 * equal phew_fill's up to the last fp32 places, where those and the
 * device's logf / sincospif round apart. */
int phew_fill_host(void* out, int64_t n, int64_t cols, int dtype, int kind, uint64_t seed,
                   uint64_t stream_id, float scale, int threads);

/* ---- equivalence comparison -------------------------------------------- */

/* Result of one baseline/candidate comparison, written to DEVICE memory. */
typedef struct phew_compare_stats {
  double sum_abs_base;      /* sum |b| over all elements (fp64, fixed order)   */
  double mean_abs_base;     /* sum_abs_base / n                                */
  double max_abs_diff;      /* max |b - c| over pairs where neither is NaN
                               (an infinite difference counts: +inf)          */
  double atol_used;         /* tolerance actually applied (after bf16 relax)   */
  double rtol_used;
  int64_t n;                /* elements compared                               */
  int64_t n_nonfinite_base; /* count of NaN/Inf in the baseline               */
  int64_t n_mismatch;       /* elements failing the allclose rule              */
  int64_t n_nan_any;        /* elements where b or c is NaN                    */
  int32_t skipped;          /* 1 = comparison skipped (non-finite baseline, or
                               bf16 with mean|b| > 1e10)                        */
  int32_t passed;           /* 1 = the allclose rule held (or skipped)         */
} phew_compare_stats;

/* Bytes of scratch phew_compare needs for n elements. */
size_t phew_compare_scratch_bytes(int64_t n);

/* Compares baseline `b` against candidate `c` (n elements of `dtype`) with
 * the rule of the reference's equivalence checker (verify/checker.py:144-209
 * and _allclose :220-233): skip when the baseline holds a non-finite value;
 * for bf16, skip when mean|b| > 1e10, else relax to atol = max(atol,
 * mean|b| * f), rtol = max(rtol, f) with f = 0.30 if mean|b| > 1e6 else 0.05;
 * pass iff NaN positions agree and |b - c| <= atol + rtol * |c| (or b == c),
 * evaluated in the arithmetic numpy uses for that dtype (fp16 math for fp16
 * outputs, fp32 otherwise).  `scratch` (device, phew_compare_scratch_bytes(n)
 * bytes, caller-owned) holds per-block partial results.  `out` is a device
 * pointer.  Deterministic: the same inputs give the same bits on any GPU. */
int phew_compare(const void* b, const void* c, int64_t n, int dtype,
                 double atol, double rtol, void* scratch, size_t scratch_bytes,
                 phew_compare_stats* out, void* stream);

/* phew_compare for callers that cannot allocate device memory when they
 * need a verdict -- code running during CUDA graph capture, inside a host
 * runtime whose allocator owns the device, or in a context that must not
 * synchronise the device (cudaMalloc/cudaFree may).  Same inputs, outputs
 * and result as phew_compare, but the per-block partials live in a
 * 48 KiB array in this library's own device memory (held by every GPU that
 * loads the library until the process exits); the call allocates nothing.
 *   - The first call on each device looks up that array's address on the
 *     current device (cudaGetSymbolAddress); make that first call before
 *     any stream capture.  The address is kept per device and per context:
 *     after a device reset (cudaDeviceReset, or a released and re-created
 *     primary context) the next call looks it up again, so that call too
 *     belongs before any capture.
 *   - Every call shares the one array: calls that overlap on the GPU (for
 *     instance on two streams at once) race.  Nothing in it needs clearing.
 *   - Comparisons whose scratch need (phew_compare_scratch_bytes) exceeds
 *     the array are refused with PHEW_ERR_INVALID.
 * No counterpart in the reference (its comparison runs in numpy on the
 * host, verify/checker.py:220-233). */
int phew_compare_static(const void* b, const void* c, int64_t n, int dtype,
                        double atol, double rtol, phew_compare_stats* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PHEW_B200_H */
