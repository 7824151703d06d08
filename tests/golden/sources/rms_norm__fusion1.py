import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, *_, **__):
    t1 = x0 * x0
    t2 = mx.mean(t1, axis=[1], keepdims=True)
    _kernel_97 = mx.fast.cuda_kernel(
        name="kernel_97",
        input_names=['inp0', 'inp1', 'inp2'],
        output_names=['out0'],
        source="""    // fused elementwise chain: 4 ops, 3 inputs, 1 outputs, 2097152 elements
    // phew-io: idx32 out=1024x2048 inp0=prefix:2048 inp1=full inp2=suffix:2048
    const unsigned int phew_n = (unsigned int)out0_size;
    const unsigned int phew_tid = (unsigned int)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned int phew_nthreads = (unsigned int)gridDim.x * blockDim.x;
    unsigned int phew_tail = 0;
    const float v4 = __int_as_float(0x3727c5ac) /* 9.999999747378752e-06 */;
    if (((reinterpret_cast<phew_uptr>(inp0) | reinterpret_cast<phew_uptr>(inp1) | reinterpret_cast<phew_uptr>(inp2) | reinterpret_cast<phew_uptr>(out0)) & 15u) == 0u) {
      const unsigned int phew_nvec = phew_n / 4u;
      for (unsigned int phew_v = phew_tid; phew_v < phew_nvec; phew_v += phew_nthreads) {
        const unsigned int elem = phew_v * 4u;
        const float ld0 = inp0[elem / 2048u];
        const phew_vec<float, 4> ld1 = phew_ldv<float, 4>(inp1 + elem);
        const phew_vec<float, 4> ld2 = phew_ldv<float, 4>(inp2 + elem % 2048u);
        phew_vec<float, 4> st0;
        #pragma unroll
        for (int l = 0; l < 4; ++l) {
          const float v1 = phew_ld(ld0);
          const float v2 = phew_ld(ld1.v[l]);
          const float v3 = phew_ld(ld2.v[l]);
          const float v5 = __fadd_rn(v1, v4);
          const float v6 = __fdiv_rn(1.0f, __fsqrt_rn(v5));
          const float v7 = __fmul_rn(v2, v6);
          const float v8 = __fmul_rn(v7, v3);
          st0.v[l] = phew_st_f32(v8);
        }
        phew_stv<float, 4>(out0 + elem, st0);
      }
      phew_tail = phew_nvec * 4u;
    }
    for (unsigned int elem = phew_tail + phew_tid; elem < phew_n; elem += phew_nthreads) {
      const float v1 = phew_ld(inp0[elem / 2048u]);
      const float v2 = phew_ld(inp1[elem]);
      const float v3 = phew_ld(inp2[elem % 2048u]);
      const float v5 = __fadd_rn(v1, v4);
      const float v6 = __fdiv_rn(1.0f, __fsqrt_rn(v5));
      const float v7 = __fmul_rn(v2, v6);
      const float v8 = __fmul_rn(v7, v3);
      out0[elem] = phew_st_f32(v8);
    }""",
    )
    kernel3_out = _kernel_97(
        inputs=[t2, x0, x1],
        output_shapes=[x0.shape],
        output_dtypes=[mx.float32],
        grid=(mx.elementwise_threads(x0.size), 1, 1),
        threadgroup=(256, 1, 1),
        template=[],
    )
    kernel3 = kernel3_out[0]
    return kernel3
