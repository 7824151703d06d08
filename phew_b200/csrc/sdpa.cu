// Scaled dot-product attention forward on the tcgen05 tensor cores.
//
//   O[b, h] = softmax(Q[b, h] K[b, h]^T * scale  (+ causal mask)) V[b, h]
//
// Stands in for mx.fast.scaled_dot_product_attention (phew emit/codegen.py:421-426,
// node FastScaledDotProductAttention ir/ops.py:182-187, matched by
// rules/primitive_subst.py:413-499) and, with causal = 1, for the naive masked
// attention graph softmax(q @ k.T * s + mask) @ v it is substituted for.
//
// Layout: Q, K, V, O are [B*H, L, D] row-major bf16/fp16 (D contiguous),
// D = 128, L a multiple of 128.  One CTA owns one (b, h, 128-row query tile)
// and streams 128-row key/value tiles through a 2-deep shared-memory ring:
//
//   warp 0     TMA: Q once, then K_j / V_j (128B-swizzled, no multicast)
//   warp 1     TMEM owner + MMA issuer:
//                S_j  = Q K_j^T  -> TMEM (two S buffers, 128 fp32 columns each)
//                O   += P_j V_j  -> TMEM (128 fp32 columns), P_j read from TMEM
//   warps 2-5  softmax, one query row per thread: scaled/masked row of S_j,
//              running max with lazy rescaling (O and the row sum are rescaled
//              only when the max grows by more than 2^8), P_j = exp2(S - max)
//              written back over S_j as packed 16-bit pairs, and the final
//              O / rowsum epilogue.
//
// All waits are bounded; a wait that runs out sets *error_flag and the CTA
// winds down (TMEM is always released).
#include "tc_common.cuh"

namespace phew {
namespace attn {

using namespace tc;

constexpr int BQ = 128;  // query rows per CTA
constexpr int BKV = 128; // key/value rows per tile
constexpr int D = 128;
constexpr int kThreads = 192;
constexpr int TILE_BYTES = BKV * D * 2;       // 32 KB: one Q, K or V tile
constexpr int HALF_BYTES = TILE_BYTES / 2;    // one 64-column swizzle half
constexpr int SMEM = TILE_BYTES * 5 + 1024 + 256;  // Q + 2 x (K, V)
constexpr int TMEM_COLS = 512;                // S0, S1 (128 each) + O (128)
constexpr int S_COL0 = 0, O_COL = 256;
constexpr float kRescaleThreshold = 8.0f;     // log2 units

struct Params {
  int L;           // sequence length (multiple of BQ)
  int bh;          // batch * heads
  int causal;
  float scale_log2;  // scale * log2(e)
  void* O;
  int out_dtype;
  int* error_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t d;
  if (BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    sdpa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + TILE_BYTES, smem + 3 * TILE_BYTES};
  uint8_t* sV[2] = {smem + 2 * TILE_BYTES, smem + 4 * TILE_BYTES};
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 5 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* o_bar = bars + 11;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qt = p.L / BQ;
  // Longest query tiles first: with a causal mask later tiles do more work.
  const int qt = p.causal ? (n_qt - 1 - static_cast<int>(blockIdx.x % n_qt)) : static_cast<int>(blockIdx.x % n_qt);
  const int bh = static_cast<int>(blockIdx.x / n_qt);
  const int q0 = qt * BQ;
  const int n_kv = p.causal ? qt + 1 : p.L / BKV;
  const int row_base = bh * p.L;  // first row of this (b, h) in the [B*H*L, D] view

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_bar[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, 0, row_base + q0);
      tma_load_2d(sQ + HALF_BYTES, &tmQ, q_full, 64, row_base + q0);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, p.error_flag)) { ok = false; break; }
        const int r = row_base + j * BKV;
        mbar_expect_tx(&k_full[s], TILE_BYTES);
        tma_load_2d(sK[s], &tmK, &k_full[s], 0, r);
        tma_load_2d(sK[s] + HALF_BYTES, &tmK, &k_full[s], 64, r);
        mbar_expect_tx(&v_full[s], TILE_BYTES);
        tma_load_2d(sV[s], &tmV, &v_full[s], 0, r);
        tma_load_2d(sV[s] + HALF_BYTES, &tmV, &v_full[s], 64, r);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_qk = instr_desc_f16(BF16 ? 1 : 0, 0, BQ, BKV);
      constexpr uint32_t id_pv = instr_desc_f16(BF16 ? 1 : 0, 1, BQ, D);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, p.error_flag)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t k_addr = smem_u32(sK[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
          mma_ss(tmem + S_COL0 + s * 128, smem_desc(q_addr + off, 16, 1024),
                 smem_desc(k_addr + off, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
        }
        commit(&s_full[s]);
        return true;
      };
      if (!mbar_wait(q_full, 0, p.error_flag)) ok = false;
      if (ok) ok = issue_s(0);
      if (ok && n_kv > 1) ok = issue_s(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&p_full[s], ph, p.error_flag) || !mbar_wait(&v_full[s], ph, p.error_flag)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t v_addr = smem_u32(sV[s]);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // P_j: 128 rows x 128 kv as packed pairs in S buffer s (8 columns per k-step)
          mma_ts(tmem + O_COL, tmem + S_COL0 + s * 128 + kk * 8,
                 smem_desc(v_addr + kk * (16 * 128), HALF_BYTES, 1024), id_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
        commit(&o_bar[s]);
        commit(&kv_empty[s]);
        if (j + 2 < n_kv) {
          // S_{j+2} reuses buffer s: wait until PV_j has consumed P_j.
          if (!mbar_wait(&o_bar[s], ph, p.error_flag)) { ok = false; break; }
          ok = issue_s(j + 2);
        }
      }
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // row within the query tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int q_idx = q0 + row;
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, p.error_flag)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t raw[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_addr + S_COL0 + s * 128 + c * 32, raw + c * 32);
      tmem_ld_wait();
      float v[128];
      const bool diag = p.causal && j == n_kv - 1;
      float m_tile = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        float x = __uint_as_float(raw[i]) * p.scale_log2;
        if (diag && (j * BKV + i) > q_idx) x = -INFINITY;
        v[i] = x;
        m_tile = fmaxf(m_tile, x);
      }
      // Lazy rescaling: keep the reference max unless the row max grew by
      // more than 2^kRescaleThreshold (or this is the first tile).
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_ref = m_tile;
      } else if (m_tile > m_ref + kRescaleThreshold) {
        alpha = ex2(m_ref - m_tile);
        m_ref = m_tile;
        rescale = true;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds PV_0..PV_{j-1}: wait for PV_{j-1}, then O *= alpha.
        const int sp = (j - 1) & 1;
        if (!mbar_wait(&o_bar[sp], ((j - 1) >> 1) & 1, p.error_flag)) { ok = false; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_addr + O_COL + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem + lane_addr + O_COL + c * 32, o);
          }
        }
      }
      l *= alpha;
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float e0 = ex2(v[2 * i] - m_ref);
        const float e1 = ex2(v[2 * i + 1] - m_ref);
        l += e0 + e1;
        pk[i] = pack2<BF16>(e0, e1);
      }
      tmem_st32(tmem + lane_addr + S_COL0 + s * 128, pk);
      tmem_st32(tmem + lane_addr + S_COL0 + s * 128 + 32, pk + 32);
      tmem_st_wait();
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    // Epilogue: O / l after the last PV.
    if (ok) {
      const int jl = n_kv - 1;
      if (!mbar_wait(&o_bar[jl & 1], (jl >> 1) & 1, p.error_flag)) ok = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      const float inv = 1.0f / l;
      uint8_t* out = static_cast<uint8_t*>(p.O) + (static_cast<long long>(row_base) + q_idx) * D * 2;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_addr + O_COL + c * 32, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(out + c * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
  }
  if (!ok && p.error_flag) atomicExch(p.error_flag, PHEW_ERR_TIMEOUT);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// [rows, 128] row-major 16-bit tensor, box = 64 columns x 128 rows, 128B swizzle.
int make_map(CUtensorMap* tm, const void* base, bool bf16, uint64_t rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(D), rows};
  const uint64_t strides[1] = {static_cast<uint64_t>(D) * 2};
  const uint32_t box[2] = {64, 128};
  return make_map_16bit(tm, base, bf16, 2, dims, strides, box);
}

template <bool BF16>
int launch(const void* q, const void* k, const void* v, const Params& p, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  const uint64_t rows = static_cast<uint64_t>(p.bh) * p.L;
  int s = make_map(&tq, q, BF16, rows);
  if (!s) s = make_map(&tk, k, BF16, rows);
  if (!s) s = make_map(&tv, v, BF16, rows);
  if (s) return s;
  static bool attr = false;
  if (!attr) {
    PHEW_CHECK_CUDA(cudaFuncSetAttribute(sdpa_fwd_kernel<BF16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr = true;
  }
  const unsigned grid = static_cast<unsigned>(p.bh) * (p.L / BQ);
  sdpa_fwd_kernel<BF16><<<grid, kThreads, SMEM, st>>>(tq, tk, tv, p);
  return launch_status("sdpa_fwd_kernel");
}

}  // namespace attn
}  // namespace phew

using namespace phew;

extern "C" int phew_sdpa_supported(int64_t L, int64_t D, int dtype) {
  return (L > 0 && L % attn::BQ == 0 && D == attn::D && (dtype == PHEW_BF16 || dtype == PHEW_F16)) ? 1 : 0;
}

extern "C" int phew_sdpa(const void* q, const void* k, const void* v, void* o, int64_t batch_heads,
                         int64_t L, int64_t D, float scale, int causal, int dtype, int* error_flag,
                         void* stream) {
  PHEW_REQUIRE(q && k && v && o, "phew_sdpa: null pointer");
  PHEW_REQUIRE(phew_sdpa_supported(L, D, dtype), "phew_sdpa: needs D == 128, L % 128 == 0, bf16/f16");
  PHEW_REQUIRE(batch_heads > 0 && batch_heads * L < (1LL << 31), "phew_sdpa: bad batch");
  PHEW_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                 reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15) == 0,
               "phew_sdpa: pointers must be 16-byte aligned");
  attn::Params p;
  p.L = static_cast<int>(L);
  p.bh = static_cast<int>(batch_heads);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.O = o;
  p.out_dtype = dtype;
  p.error_flag = error_flag;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == PHEW_BF16 ? attn::launch<true>(q, k, v, p, st) : attn::launch<false>(q, k, v, p, st);
}
