import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, *_, **__):
    t1 = x0[:, :, :, :64]
    t2 = x0[:, :, :, 64:]
    _kernel_251 = mx.fast.cuda_kernel(
        name="kernel_251",
        input_names=['inp0', 'inp1', 'inp2'],
        output_names=['out0', 'out1'],
        source="""    // fused elementwise chain: 8 ops, 3 inputs, 2 outputs, 33554432 elements
    // phew-io: idx32 out=8x32x2048x64 inp0=suffix:131072 inp1=full inp2=full
    const unsigned int phew_n = (unsigned int)out0_size;
    const unsigned int phew_tid = (unsigned int)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned int phew_nthreads = (unsigned int)gridDim.x * blockDim.x;
    unsigned int phew_tail = 0;
    if (((reinterpret_cast<phew_uptr>(inp0) | reinterpret_cast<phew_uptr>(inp1) | reinterpret_cast<phew_uptr>(inp2) | reinterpret_cast<phew_uptr>(out0) | reinterpret_cast<phew_uptr>(out1)) & 15u) == 0u) {
      const unsigned int phew_nvec = phew_n / 8u;
      for (unsigned int phew_v = phew_tid; phew_v < phew_nvec; phew_v += phew_nthreads) {
        const unsigned int elem = phew_v * 8u;
        const phew_vec<phew_bf16, 8> ld0 = phew_ldv<phew_bf16, 8>(inp0 + elem % 131072u);
        const phew_vec<phew_bf16, 8> ld1 = phew_ldv<phew_bf16, 8>(inp1 + elem);
        const phew_vec<phew_bf16, 8> ld2 = phew_ldv<phew_bf16, 8>(inp2 + elem);
        phew_vec<phew_bf16, 8> st0;
        phew_vec<phew_bf16, 8> st1;
        #pragma unroll
        for (int p = 0; p < 4; ++p) {
          const phew_u32 v1 = phew_pair(ld0, p);
          const phew_u32 v2 = phew_pair(ld1, p);
          const phew_u32 v3 = phew_pair(ld2, p);
          const phew_u32 v4 = phew_b2_pack(cosf(phew_b2_lo(v1)), cosf(phew_b2_hi(v1)));
          const phew_u32 v5 = phew_b2_mul(v2, v4);
          const phew_u32 v6 = phew_b2_pack(sinf(phew_b2_lo(v1)), sinf(phew_b2_hi(v1)));
          const phew_u32 v7 = phew_b2_mul(v3, v6);
          const phew_u32 v8 = phew_b2_sub(v5, v7);
          const phew_u32 v9 = phew_b2_mul(v2, v6);
          const phew_u32 v10 = phew_b2_mul(v3, v4);
          const phew_u32 v11 = phew_b2_add(v9, v10);
          phew_set_pair(st0, p, v8);
          phew_set_pair(st1, p, v11);
        }
        phew_stv<phew_bf16, 8>(out0 + elem, st0);
        phew_stv<phew_bf16, 8>(out1 + elem, st1);
      }
      phew_tail = phew_nvec * 8u;
    }
    for (unsigned int elem = phew_tail + phew_tid; elem < phew_n; elem += phew_nthreads) {
      const float v1 = phew_ld(inp0[elem % 131072u]);
      const float v2 = phew_ld(inp1[elem]);
      const float v3 = phew_ld(inp2[elem]);
      const float v4 = phew_rnd_bf16(cosf(v1));
      const float v5 = phew_rnd_bf16(__fmul_rn(v2, v4));
      const float v6 = phew_rnd_bf16(sinf(v1));
      const float v7 = phew_rnd_bf16(__fmul_rn(v3, v6));
      const float v8 = phew_rnd_bf16(__fsub_rn(v5, v7));
      const float v9 = phew_rnd_bf16(__fmul_rn(v2, v6));
      const float v10 = phew_rnd_bf16(__fmul_rn(v3, v4));
      const float v11 = phew_rnd_bf16(__fadd_rn(v9, v10));
      out0[elem] = phew_st_bf16(v8);
      out1[elem] = phew_st_bf16(v11);
    }""",
    )
    kernel3_out = _kernel_251(
        inputs=[x1, t1, t2],
        output_shapes=[(8, 32, 2048, 64), (8, 32, 2048, 64)],
        output_dtypes=[mx.bfloat16, mx.bfloat16],
        grid=(33554432, 1, 1),
        threadgroup=(256, 1, 1),
        template=[],
    )
    t4 = kernel3_out[0]
    t5 = kernel3_out[1]
    t6 = mx.concatenate([t4, t5], axis=3)
    return t6
