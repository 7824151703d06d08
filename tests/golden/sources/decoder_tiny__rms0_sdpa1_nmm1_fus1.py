import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, x4, x5, x6, x7, *_, **__):
    t1 = x0 * x0
    t2 = mx.mean(t1, axis=[2], keepdims=True)
    _kernel_1452 = mx.fast.cuda_kernel(
        name="kernel_1452",
        input_names=['inp0', 'inp1', 'inp2'],
        output_names=['out0'],
        source="""    // fused elementwise chain: 4 ops, 3 inputs, 1 outputs, 131072 elements
    // phew-io: idx32 out=2x256x256 inp0=prefix:256 inp1=full inp2=suffix:256
    const unsigned int phew_n = (unsigned int)out0_size;
    const unsigned int phew_tid = (unsigned int)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned int phew_nthreads = (unsigned int)gridDim.x * blockDim.x;
    unsigned int phew_tail = 0;
    const float v4 = __int_as_float(0x37280000) /* 1.0013580322265625e-05 */;
    const phew_u32 v4_x2 = 0x37283728u;
    if (((reinterpret_cast<phew_uptr>(inp0) | reinterpret_cast<phew_uptr>(inp1) | reinterpret_cast<phew_uptr>(inp2) | reinterpret_cast<phew_uptr>(out0)) & 15u) == 0u) {
      const unsigned int phew_nvec = phew_n / 8u;
      for (unsigned int phew_v = phew_tid; phew_v < phew_nvec; phew_v += phew_nthreads) {
        const unsigned int elem = phew_v * 8u;
        const phew_bf16 ld0 = inp0[elem / 256u];
        const phew_vec<phew_bf16, 8> ld1 = phew_ldv<phew_bf16, 8>(inp1 + elem);
        const phew_vec<phew_bf16, 8> ld2 = phew_ldv<phew_bf16, 8>(inp2 + elem % 256u);
        phew_vec<phew_bf16, 8> st0;
        #pragma unroll
        for (int p = 0; p < 4; ++p) {
          const phew_u32 v1 = phew_splat2(ld0);
          const phew_u32 v2 = phew_pair(ld1, p);
          const phew_u32 v3 = phew_pair(ld2, p);
          const phew_u32 v5 = phew_b2_add(v1, v4_x2);
          const phew_u32 v6 = phew_b2_pack(__fdiv_rn(1.0f, __fsqrt_rn(phew_b2_lo(v5))), __fdiv_rn(1.0f, __fsqrt_rn(phew_b2_hi(v5))));
          const phew_u32 v7 = phew_b2_mul(v2, v6);
          const phew_u32 v8 = phew_b2_mul(v7, v3);
          phew_set_pair(st0, p, v8);
        }
        phew_stv<phew_bf16, 8>(out0 + elem, st0);
      }
      phew_tail = phew_nvec * 8u;
    }
    for (unsigned int elem = phew_tail + phew_tid; elem < phew_n; elem += phew_nthreads) {
      const float v1 = phew_ld(inp0[elem / 256u]);
      const float v2 = phew_ld(inp1[elem]);
      const float v3 = phew_ld(inp2[elem % 256u]);
      const float v5 = phew_rnd_bf16(__fadd_rn(v1, v4));
      const float v6 = phew_rnd_bf16(__fdiv_rn(1.0f, __fsqrt_rn(v5)));
      const float v7 = phew_rnd_bf16(__fmul_rn(v2, v6));
      const float v8 = phew_rnd_bf16(__fmul_rn(v7, v3));
      out0[elem] = phew_st_bf16(v8);
    }""",
    )
    kernel3_out = _kernel_1452(
        inputs=[t2, x0, x1],
        output_shapes=[x0.shape],
        output_dtypes=[mx.bfloat16],
        grid=(mx.elementwise_threads(x0.size), 1, 1),
        threadgroup=(256, 1, 1),
        template=[],
    )
    kernel3 = kernel3_out[0]
    t4 = kernel3 @ x2
    t5 = mx.reshape(t4, [t4.shape[0], t4.shape[1], 3, 2, 128])
    t6 = mx.transpose(t5, [2, 0, 3, 1, 4])
    t7 = t6[0]
    t8 = t6[1]
    t9 = t6[2]
    t10 = mx.fast.scaled_dot_product_attention(t7, t8, t9, scale=0.08838834764831843)
    t11 = mx.transpose(t10, [0, 2, 1, 3])
    t12 = mx.reshape(t11, [t11.shape[0], t11.shape[1], -1])
    t13 = t12 @ x3
    t14 = x0 + t13
    t15 = mx.fast.scaled_dot_product_attention(t12, x3, x6, scale=1.0)
    t16 = t14 + t15
    return t16
