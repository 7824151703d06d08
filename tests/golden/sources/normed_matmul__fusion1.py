import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, *_, **__):
    t1 = x0 * x0
    t2 = mx.mean(t1, axis=[1], keepdims=True)
    t3 = x0 @ x1
    _kernel_193 = mx.fast.cuda_kernel(
        name="kernel_193",
        input_names=['inp0', 'inp1'],
        output_names=['out0'],
        source="""    // fused elementwise chain: 3 ops, 2 inputs, 1 outputs, 33554432 elements
    // phew-io: idx32 out=8192x4096 inp0=prefix:4096 inp1=full
    const unsigned int phew_n = (unsigned int)out0_size;
    const unsigned int phew_tid = (unsigned int)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned int phew_nthreads = (unsigned int)gridDim.x * blockDim.x;
    unsigned int phew_tail = 0;
    const float v3 = __int_as_float(0x37280000) /* 1.0013580322265625e-05 */;
    const phew_u32 v3_x2 = 0x37283728u;
    if (((reinterpret_cast<phew_uptr>(inp0) | reinterpret_cast<phew_uptr>(inp1) | reinterpret_cast<phew_uptr>(out0)) & 15u) == 0u) {
      const unsigned int phew_nvec = phew_n / 8u;
      for (unsigned int phew_v = phew_tid; phew_v < phew_nvec; phew_v += phew_nthreads) {
        const unsigned int elem = phew_v * 8u;
        const phew_bf16 ld0 = inp0[elem / 4096u];
        const phew_vec<phew_bf16, 8> ld1 = phew_ldv<phew_bf16, 8>(inp1 + elem);
        phew_vec<phew_bf16, 8> st0;
        #pragma unroll
        for (int p = 0; p < 4; ++p) {
          const phew_u32 v1 = phew_splat2(ld0);
          const phew_u32 v2 = phew_pair(ld1, p);
          const phew_u32 v4 = phew_b2_add(v1, v3_x2);
          const phew_u32 v5 = phew_b2_pack(__fdiv_rn(1.0f, __fsqrt_rn(phew_b2_lo(v4))), __fdiv_rn(1.0f, __fsqrt_rn(phew_b2_hi(v4))));
          const phew_u32 v6 = phew_b2_mul(v2, v5);
          phew_set_pair(st0, p, v6);
        }
        phew_stv<phew_bf16, 8>(out0 + elem, st0);
      }
      phew_tail = phew_nvec * 8u;
    }
    for (unsigned int elem = phew_tail + phew_tid; elem < phew_n; elem += phew_nthreads) {
      const float v1 = phew_ld(inp0[elem / 4096u]);
      const float v2 = phew_ld(inp1[elem]);
      const float v4 = phew_rnd_bf16(__fadd_rn(v1, v3));
      const float v5 = phew_rnd_bf16(__fdiv_rn(1.0f, __fsqrt_rn(v4)));
      const float v6 = phew_rnd_bf16(__fmul_rn(v2, v5));
      out0[elem] = phew_st_bf16(v6);
    }""",
    )
    kernel4_out = _kernel_193(
        inputs=[t2, t3],
        output_shapes=[t3.shape],
        output_dtypes=[mx.bfloat16],
        grid=(mx.elementwise_threads(t3.size), 1, 1),
        threadgroup=(256, 1, 1),
        template=[],
    )
    kernel4 = kernel4_out[0]
    return kernel4
