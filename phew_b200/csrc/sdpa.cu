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
// D = 128, L a multiple of 128.  One CTA owns two 128-row query tiles (a and
// b, 256 consecutive query rows) of one (b, h), so every 128-row key/value
// tile it loads serves two S = Q K^T and two O += P V products.  Key and value
// tiles stream through separate 2-deep shared-memory rings: a key tile is
// released as soon as both S products that read it are done, a value tile
// after both P V products, so the next loads start early.
//
//   warp 0      TMA: Q_a, Q_b once, then K_j and V_j (128B-swizzled, no multicast)
//   warp 1      TMEM owner + MMA issuer, per key tile j:
//                 O_a += P_a V_j, O_b += P_b V_j        (P from TMEM)
//                 S_a  = Q_a K_{j+1}^T, S_b = Q_b K_{j+1}^T
//               so the softmax of one query tile overlaps the products of
//               the other, and each wait for a finished product is covered
//               by the other tile's product still running.
//   warps 2-5   softmax of tile a, warps 6-9 softmax of tile b, one query row
//               per thread: masked row max, running max with lazy rescaling
//               (O and the row sum are rescaled only when the max grows by
//               more than 2^8), P = exp2(S*scale*log2e - max) written back over
//               S as packed 16-bit pairs, and the final O / rowsum epilogue.
//               A quarter of the exponentials run on the FMA pipe (a cubic
//               for 2^f after rounding off the integer part) so that the
//               transcendental unit is not the limit.
//
// TMEM (512 columns): S_a 0..127, S_b 128..255, O_a 256..383, O_b 384..511.
// All waits are bounded; a wait that runs out sets *error_flag and the CTA
// winds down (TMEM is always released).
#include "tc_common.cuh"

namespace phew {
namespace attn {

using namespace tc;

constexpr int BQ = 128;   // rows per query tile
constexpr int QT = 2;     // query tiles per CTA
constexpr int BKV = 128;  // key/value rows per tile
constexpr int D = 128;
constexpr int kThreads = 32 * (2 + 4 * QT);   // TMA, MMA, 4 softmax warps per query tile
constexpr int TILE_BYTES = BKV * D * 2;       // 32 KB: one Q, K or V tile
constexpr int HALF_BYTES = TILE_BYTES / 2;    // one 64-column swizzle half
constexpr int SMEM_TILES = QT + 2 + 2;        // Q_a, Q_b, K ring, V ring
constexpr int SMEM = TILE_BYTES * SMEM_TILES + 1024 + 256;
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0, O_COL = 256;         // + 128 * tile
constexpr float kRescaleThreshold = 8.0f;     // log2 units

struct Params {
  int L;           // sequence length (multiple of BQ)
  int bh;          // batch * heads
  int causal;
  float scale_log2;  // scale * log2(e), > 0
  void* O;
  int* error_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe for x <= 8: x = j + f with j = round(x) and f in
// [-0.5, 0.5]; 2^f by a cubic whose coefficients minimise the relative error
// on that interval (fitted by iteratively reweighted least squares; max
// relative error 7.5e-5, below half an ulp of the 16-bit P it feeds), times
// 2^j built in the exponent field.  Adding 1.5 * 2^23 rounds x to an integer
// held in the low mantissa bits (1.5 * 2^23 has zero low bits, so the
// exponent field of 2^j is (bits(t) + 127) << 23).  x is clamped at -127,
// where 2^j becomes +0: masked (-inf) scores give exactly 0, as the
// flush-to-zero ex2.approx does; NaN passes through the clamp and the product.
__device__ __forceinline__ float ex2_fma(float x) {
  x = x < -127.0f ? -127.0f : x;
  const float t = __fadd_rn(x, 12582912.0f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.0f));
  float p = fmaf(0.0551716648f, f, 0.242611125f);
  p = fmaf(p, f, 0.693260968f);
  p = fmaf(p, f, 0.999928057f);
  return p * __int_as_float((__float_as_int(t) + 127) << 23);
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
  uint8_t* sQ = smem;                                  // [QT] tiles
  uint8_t* sK = smem + QT * TILE_BYTES;                // [2] tiles
  uint8_t* sV = smem + (QT + 2) * TILE_BYTES;          // [2] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_TILES * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [QT]: S_t written
  uint64_t* p_full = bars + 11;   // [QT]: P_t written (4 warps)
  uint64_t* o_done = bars + 13;   // [QT]: O_t += P_t V done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qb = (p.L + BQ * QT - 1) / (BQ * QT);
  // Longest query blocks first across the whole grid: with a causal mask
  // later blocks do more work, and finishing them first evens out the tail.
  const int qb = p.causal ? (n_qb - 1 - static_cast<int>(blockIdx.x / p.bh)) : static_cast<int>(blockIdx.x / p.bh);
  const int bh = static_cast<int>(blockIdx.x % p.bh);
  const int q0 = qb * BQ * QT;
  const int row_base = bh * p.L;  // first row of this (b, h) in the [B*H*L, D] view
  const int n_tiles = (q0 + BQ < p.L) ? 2 : 1;
  // key tiles each query tile needs (0 for a missing tile b)
  const int n_kv_a = p.causal ? q0 / BKV + 1 : p.L / BKV;
  const int n_kv_b = n_tiles == 2 ? (p.causal ? n_kv_a + 1 : n_kv_a) : 0;
  const int n_kv_max = n_tiles == 2 ? n_kv_b : n_kv_a;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
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
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(q_full, TILE_BYTES * n_tiles);
      for (int t = 0; t < n_tiles; ++t) {
        tma_load_2d(sQ + t * TILE_BYTES, &tmQ, q_full, 0, row_base + q0 + t * BQ);
        tma_load_2d(sQ + t * TILE_BYTES + HALF_BYTES, &tmQ, q_full, 64, row_base + q0 + t * BQ);
      }
      for (int j = 0; j < n_kv_max && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        const int r = row_base + j * BKV;
        if (!mbar_wait(&k_empty[s], ph, p.error_flag)) { ok = false; break; }
        mbar_expect_tx(&k_full[s], TILE_BYTES);
        tma_load_2d(sK + s * TILE_BYTES, &tmK, &k_full[s], 0, r);
        tma_load_2d(sK + s * TILE_BYTES + HALF_BYTES, &tmK, &k_full[s], 64, r);
        if (!mbar_wait(&v_empty[s], ph, p.error_flag)) { ok = false; break; }
        mbar_expect_tx(&v_full[s], TILE_BYTES);
        tma_load_2d(sV + s * TILE_BYTES, &tmV, &v_full[s], 0, r);
        tma_load_2d(sV + s * TILE_BYTES + HALF_BYTES, &tmV, &v_full[s], 64, r);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_qk = instr_desc_f16(BF16 ? 1 : 0, 0, BQ, BKV);
      constexpr uint32_t id_pv = instr_desc_f16(BF16 ? 1 : 0, 1, BQ, D);
      // S_t = Q_t K_j^T for every tile that still needs key tile j.
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, p.error_flag)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t k_addr = smem_u32(sK + s * TILE_BYTES);
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (j >= (t == 0 ? n_kv_a : n_kv_b)) continue;
          // S_t still holds P_t of tile j-1 until O_t += P_t V_{j-1} is done.
          if (j > 0 && !mbar_wait(&o_done[t], (j - 1) & 1, p.error_flag)) return false;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t q_addr = smem_u32(sQ + t * TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
            mma_ss(tmem + S_COL + t * 128, smem_desc(q_addr + off, 16, 1024),
                   smem_desc(k_addr + off, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
          }
          commit(&s_full[t]);
        }
        commit(&k_empty[s]);
        return true;
      };
      if (!mbar_wait(q_full, 0, p.error_flag)) ok = false;
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv_max && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, p.error_flag)) { ok = false; break; }
        const uint32_t v_addr = smem_u32(sV + s * TILE_BYTES);
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (!ok || j >= (t == 0 ? n_kv_a : n_kv_b)) continue;
          if (!mbar_wait(&p_full[t], j & 1, p.error_flag)) { ok = false; continue; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            // P_t: 128 rows x 128 keys as packed pairs in S_t (8 columns per k-step)
            mma_ts(tmem + O_COL + t * 128, tmem + S_COL + t * 128 + kk * 8,
                   smem_desc(v_addr + kk * (16 * 128), HALF_BYTES, 1024), id_pv,
                   (j > 0 || kk > 0) ? 1u : 0u);
          }
          commit(&o_done[t]);
        }
        if (!ok) break;
        commit(&v_empty[s]);
        if (j + 1 < n_kv_max) ok = issue_s(j + 1);
      }
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..9) ----------------
    const int t = (warp - 2) >> 2;        // query tile
    const int quarter = warp & 3;         // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;  // row within the query tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + S_COL + t * 128;
    const uint32_t o_addr = tmem + lane_addr + O_COL + t * 128;
    const int q_idx = q0 + t * BQ + row;
    const int nkv = t == 0 ? n_kv_a : n_kv_b;
    const float c = p.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < nkv && ok; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, p.error_flag)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t raw[128];
#pragma unroll
      for (int k = 0; k < 4; ++k) tmem_ld32(s_addr + k * 32, raw + k * 32);
      tmem_ld_wait();
      if (p.causal && j == nkv - 1) {
        // diagonal tile: key j*BKV + i is visible to row q_idx iff i <= row
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > row) raw[i] = __float_as_uint(-INFINITY);
      }
      // The row max over unscaled scores (scale > 0), then scaled.
      float mx = __uint_as_float(raw[0]);
#pragma unroll
      for (int i = 1; i < 128; ++i) mx = fmaxf(mx, __uint_as_float(raw[i]));
      const float m_tile = mx * c;
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
      l *= alpha;
      const float neg_m = -m_ref;
      // P in two halves of 64 keys (32 packed columns each), so that only
      // 32 packed registers are live beside the scores.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x0 = fmaf(__uint_as_float(raw[64 * h + 2 * i]), c, neg_m);
          const float x1 = fmaf(__uint_as_float(raw[64 * h + 2 * i + 1]), c, neg_m);
          float e0, e1;
          if ((i & 3) == 3) {
            e0 = ex2_fma(x0);
            e1 = ex2_fma(x1);
          } else {
            e0 = ex2(x0);
            e1 = ex2(x1);
          }
          l += e0 + e1;
          pk[i] = pack2<BF16>(e0, e1);
        }
        tmem_st32(s_addr + 32 * h, pk);
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // O_t holds the products of tiles 0..j-1: wait for the last one.
        // (Done after P is written, when the scores are no longer live.)
        if (!mbar_wait(&o_done[t], (j - 1) & 1, p.error_flag)) ok = false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t o[32];
            tmem_ld32(o_addr + k * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_addr + k * 32, o);
          }
        }
      }
      tmem_st_wait();
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // Epilogue: O_t / l after the last product.
    if (ok && nkv > 0 && !mbar_wait(&o_done[t], (nkv - 1) & 1, p.error_flag)) ok = false;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && nkv > 0) {
      const float inv = 1.0f / l;
      uint8_t* out = static_cast<uint8_t*>(p.O) + (static_cast<long long>(row_base) + q_idx) * D * 2;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t o[32];
        tmem_ld32(o_addr + k * 32, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(out + k * 64);
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
  const unsigned grid = static_cast<unsigned>(p.bh) * ((p.L + BQ * QT - 1) / (BQ * QT));
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
  // The row max is taken over the unscaled scores.
  PHEW_REQUIRE(scale > 0.0f, "phew_sdpa: scale must be positive");
  PHEW_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                 reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15) == 0,
               "phew_sdpa: pointers must be 16-byte aligned");
  attn::Params p;
  p.L = static_cast<int>(L);
  p.bh = static_cast<int>(batch_heads);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.O = o;
  p.error_flag = error_flag;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == PHEW_BF16 ? attn::launch<true>(q, k, v, p, st) : attn::launch<false>(q, k, v, p, st);
}
