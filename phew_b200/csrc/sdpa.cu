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
//   warp 0      TMA: Q_a and K_0 first (all that S_a(0) needs; issued by
//               the thread that initialises the barriers, before the block
//               sync and the TMEM allocation), then Q_b, then K_j and V_j
//               (128B-swizzled, each CTA loading its own tiles); Q_a and Q_b
//               land on separate barriers; the three tensor maps are
//               prefetched at entry
//   warp 1      TMEM owner + MMA issuer.  Per key tile j and query tile t:
//                 O_t += P_t V_j, then (once that product has read P_t out of
//                 S_t) S_t = Q_t K_{j+1}^T, so the softmax of tile a runs
//                 while the tensor pipe works for tile b and the other way
//                 round.
//   warps 2-5   softmax of tile a, warps 6-9 softmax of tile b, one query row
//               per thread: masked row max, running max with lazy rescaling
//               (O and the row sum are rescaled only when the max grows by
//               more than 2^8), P = exp2(S*scale*log2e - max) written back over
//               S as packed 16-bit pairs, and the final O / rowsum epilogue.
//               Past the first key tile P is computed against the running
//               max while the tile max is still being reduced, and redone in
//               the rare case that the max grew past the threshold.  The
//               scale/shift and the row sum run on pairs of scores (packed
//               f32x2 FMA), so each warp issues fewer instructions per score.
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
  int heads;       // (b, h) = (bh / heads, bh % heads): the q / k / v maps are [b][h][L][D] views
  int causal;
  float scale_log2;  // scale * log2(e), > 0
  void* O;
  int* error_flag;
  unsigned long long wait_ns;  // bound of every pipeline wait
  int withhold;                // test hook: the V load of key tile `withhold` is left unissued (-1: none)
};

// ---- scalar and packed (f32x2) arithmetic helpers ----
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a, b, c); like fmaxf a NaN operand is ignored.  (A NaN score still
// poisons its row: exp2 of it is NaN and so is the row sum.)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

// P = exp2(raw * c - m) over one row of 128 scores, packed into 64 16-bit
// pairs and stored to TMEM at s_addr (columns 0..63 of the S buffer).
// Returns the row sum of this tile's (unrounded) P.
template <bool BF16>
__device__ __forceinline__ float compute_p(const uint32_t* raw, float c, float m, uint32_t s_addr) {
  const uint64_t c2 = f2(c, c), nm2 = f2(-m, -m);
  uint64_t l2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int pi = 16 * h + i;
      const uint64_t x = fma2(f2(__uint_as_float(raw[2 * pi]), __uint_as_float(raw[2 * pi + 1])), c2, nm2);
      const uint64_t e = f2(ex2(lo_of(x)), ex2(hi_of(x)));
      l2[i & 1] = add2(l2[i & 1], e);
      pk[i] = pack2<BF16>(lo_of(e), hi_of(e));
    }
    tmem_st16(s_addr + 16 * h, pk);
  }
  const uint64_t l = add2(l2[0], l2[1]);
  return lo_of(l) + hi_of(l);
}

// max over 128 scores: eight independent chains of three-input max.
__device__ __forceinline__ float row_max(const uint32_t* raw) {
  float m8[8];
#pragma unroll
  for (int a = 0; a < 8; ++a)
    m8[a] = max3(__uint_as_float(raw[3 * a]), __uint_as_float(raw[3 * a + 1]), __uint_as_float(raw[3 * a + 2]));
#pragma unroll
  for (int i = 24; i + 16 <= 128; i += 16)
#pragma unroll
    for (int a = 0; a < 8; ++a)
      m8[a] = max3(m8[a], __uint_as_float(raw[i + 2 * a]), __uint_as_float(raw[i + 2 * a + 1]));
#pragma unroll
  for (int a = 0; a < 8; ++a) m8[a] = fmaxf(m8[a], __uint_as_float(raw[120 + a]));
  return max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
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
  uint64_t* q_full_b = bars + 15;  // Q_b landed (q_full: Q_a)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  uint64_t* drain = bars + 17;     // the MMA thread's last commit (failure path)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
  }
  const int n_qb = (p.L + BQ * QT - 1) / (BQ * QT);
  // CTA order: heads in groups of 16, so the CTAs running at one time share
  // the K / V of few heads in L2.  With a causal mask later query blocks do
  // more work, so within a group the longest go first (evens out the tail);
  // without one a head's query blocks run side by side.
  int qb, bh;
  if (p.causal) {
    const int G = p.bh < 16 ? p.bh : 16;
    const int grp = static_cast<int>(blockIdx.x) / (G * n_qb);
    const int rem = static_cast<int>(blockIdx.x) % (G * n_qb);
    const int gsize = (grp + 1) * G <= p.bh ? G : p.bh - grp * G;
    qb = n_qb - 1 - rem / gsize;
    bh = grp * G + rem % gsize;
  } else {
    qb = static_cast<int>(blockIdx.x % n_qb);
    bh = static_cast<int>(blockIdx.x / n_qb);
  }
  const int q0 = qb * BQ * QT;
  const int row_base = bh * p.L;  // first row of this (b, h) in the contiguous [B*H*L, D] output
  const int hh = bh % p.heads, bb = bh / p.heads;  // operand map coordinates of this (b, h)
  const int n_tiles = (q0 + BQ < p.L) ? 2 : 1;
  // key tiles each query tile needs (0 for a missing tile b)
  const int n_kv_a = p.causal ? q0 / BKV + 1 : p.L / BKV;
  const int n_kv_b = n_tiles == 2 ? (p.causal ? n_kv_a + 1 : n_kv_a) : 0;
  const int n_kv_max = n_tiles == 2 ? n_kv_b : n_kv_a;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_full_b, 1);
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
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // This thread is also the TMA producer: start Q_a and K_0 now, before
    // the block-wide sync and the TMEM allocation.
    mbar_expect_tx(q_full, TILE_BYTES);
    tma_load_4d(sQ, &tmQ, q_full, 0, q0, hh, bb);
    tma_load_4d(sQ + HALF_BYTES, &tmQ, q_full, 64, q0, hh, bb);
    mbar_expect_tx(&k_full[0], TILE_BYTES);
    tma_load_4d(sK, &tmK, &k_full[0], 0, 0, hh, bb);
    tma_load_4d(sK + HALF_BYTES, &tmK, &k_full[0], 64, 0, hh, bb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  // producer: the key tile whose K / V load each ring slot received last (-1: none)
  int k_last0 = 0, k_last1 = -1, v_last0 = -1, v_last1 = -1;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // Q_a and K_0 were issued at set-up (all that S_a(0) needs); now Q_b,
      // then the rings.
      if (n_tiles == 2) {
        mbar_expect_tx(q_full_b, TILE_BYTES);
        tma_load_4d(sQ + TILE_BYTES, &tmQ, q_full_b, 0, q0 + BQ, hh, bb);
        tma_load_4d(sQ + TILE_BYTES + HALF_BYTES, &tmQ, q_full_b, 64, q0 + BQ, hh, bb);
      }
      for (int j = 0; j < n_kv_max && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        const int r = j * BKV;  // key row within this (b, h)
        if (j > 0) {
          if (!mbar_wait(&k_empty[s], ph, p.error_flag, p.wait_ns)) { ok = false; break; }
          mbar_expect_tx(&k_full[s], TILE_BYTES);
          tma_load_4d(sK + s * TILE_BYTES, &tmK, &k_full[s], 0, r, hh, bb);
          tma_load_4d(sK + s * TILE_BYTES + HALF_BYTES, &tmK, &k_full[s], 64, r, hh, bb);
          if (s) k_last1 = j; else k_last0 = j;
        }
        if (!mbar_wait(&v_empty[s], ph, p.error_flag, p.wait_ns)) { ok = false; break; }
        if (j == p.withhold) continue;  // test hook: this V tile never lands
        if (s) v_last1 = j; else v_last0 = j;
        mbar_expect_tx(&v_full[s], TILE_BYTES);
        tma_load_4d(sV + s * TILE_BYTES, &tmV, &v_full[s], 0, r, hh, bb);
        tma_load_4d(sV + s * TILE_BYTES + HALF_BYTES, &tmV, &v_full[s], 64, r, hh, bb);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_qk = instr_desc_f16(BF16 ? 1 : 0, 0, BQ, BKV);
      constexpr uint32_t id_pv = instr_desc_f16(BF16 ? 1 : 0, 1, BQ, D);
      auto issue_s = [&](int t, uint32_t k_addr) {
        const uint32_t q_addr = smem_u32(sQ + t * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
          mma_ss(tmem + S_COL + t * 128, smem_desc(q_addr + off, 16, 1024),
                 smem_desc(k_addr + off, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
        }
        commit(&s_full[t]);
      };
      if (!mbar_wait(q_full, 0, p.error_flag, p.wait_ns) || !mbar_wait(&k_full[0], 0, p.error_flag, p.wait_ns)) ok = false;
      if (ok) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        issue_s(0, smem_u32(sK));
        if (n_tiles == 2) {
          if (!mbar_wait(q_full_b, 0, p.error_flag, p.wait_ns)) ok = false;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          if (ok) issue_s(1, smem_u32(sK));
        }
        commit(&k_empty[0]);
      }
      for (int j = 0; j < n_kv_max && ok; ++j) {
        const int s = j & 1, s1 = (j + 1) & 1;
        const bool more = j + 1 < n_kv_max;
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, p.error_flag, p.wait_ns)) { ok = false; break; }
        if (more && !mbar_wait(&k_full[s1], ((j + 1) >> 1) & 1, p.error_flag, p.wait_ns)) { ok = false; break; }
        const uint32_t v_addr = smem_u32(sV + s * TILE_BYTES);
        const uint32_t k_addr = smem_u32(sK + s1 * TILE_BYTES);
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          const int nk = t == 0 ? n_kv_a : n_kv_b;
          if (!ok || j >= nk) continue;
          if (!mbar_wait(&p_full[t], j & 1, p.error_flag, p.wait_ns)) { ok = false; continue; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            // P_t: 128 rows x 128 keys as packed pairs in S_t (8 columns per k-step)
            mma_ts(tmem + O_COL + t * 128, tmem + S_COL + t * 128 + kk * 8,
                   smem_desc(v_addr + kk * (16 * 128), HALF_BYTES, 1024), id_pv,
                   (j > 0 || kk > 0) ? 1u : 0u);
          }
          commit(&o_done[t]);
          if (j + 1 < nk) {
            // S_t holds P_t until this product has read it.
            if (!mbar_wait(&o_done[t], j & 1, p.error_flag, p.wait_ns)) { ok = false; continue; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            issue_s(t, k_addr);
          }
        }
        if (!ok) break;
        commit(&v_empty[s]);
        if (more) commit(&k_empty[s1]);
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
      if (!mbar_wait(&s_full[t], j & 1, p.error_flag, p.wait_ns)) { ok = false; break; }
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
      float tile_sum;
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_ref = row_max(raw) * c;  // raw scores are unscaled; scale > 0
        tile_sum = compute_p<BF16>(raw, c, m_ref, s_addr);
      } else {
        // P against the running max while the tile max is reduced; the max
        // only decides whether this tile must be redone.
        tile_sum = compute_p<BF16>(raw, c, m_ref, s_addr);
        const float m_tile = row_max(raw) * c;
        // Lazy rescaling: keep the running max unless the tile max exceeds
        // it by more than 2^kRescaleThreshold.
        if (m_tile > m_ref + kRescaleThreshold) {
          alpha = ex2(m_ref - m_tile);
          m_ref = m_tile;
          rescale = true;
        }
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // Redo P with the new max (rows that kept theirs recompute the same
        // values), then scale O_t, which holds the products of tiles
        // 0..j-1: wait for the last one first.
        tmem_st_wait();
        tile_sum = compute_p<BF16>(raw, c, m_ref, s_addr);
        if (!mbar_wait(&o_done[t], (j - 1) & 1, p.error_flag, p.wait_ns)) ok = false;
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
      l = fmaf(l, alpha, tile_sum);
      tmem_st_wait();
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // Epilogue: O_t / l after the last product.
    if (ok && nkv > 0 && !mbar_wait(&o_done[t], (nkv - 1) & 1, p.error_flag, p.wait_ns)) ok = false;
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
  if (__syncthreads_or(!ok)) {
    // A wait ran out somewhere in the CTA: before the shared memory and the
    // TMEM are given back, let the work still in flight land (each wait
    // bounded again): the Q tiles and the last K / V load of each ring
    // slot, and the MMAs the issuer committed.
    if (warp == 0 && lane == 0) {
      mbar_wait(q_full, 0, nullptr, p.wait_ns);
      if (n_tiles == 2) mbar_wait(q_full_b, 0, nullptr, p.wait_ns);
      if (k_last0 >= 0) mbar_wait(&k_full[0], (k_last0 >> 1) & 1, nullptr, p.wait_ns);
      if (k_last1 >= 0) mbar_wait(&k_full[1], (k_last1 >> 1) & 1, nullptr, p.wait_ns);
      if (v_last0 >= 0) mbar_wait(&v_full[0], (v_last0 >> 1) & 1, nullptr, p.wait_ns);
      if (v_last1 >= 0) mbar_wait(&v_full[1], (v_last1 >> 1) & 1, nullptr, p.wait_ns);
    } else if (warp == 1 && lane == 0) {
      commit(drain);
      mbar_wait(drain, 0, nullptr, p.wait_ns);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// [batch][heads][L][128] 16-bit view: rows `st[0]` elements apart, heads
// st[1], batches st[2]; box = 64 columns x 128 rows of one (b, h), 128B
// swizzle.
int make_map(CUtensorMap* tm, const void* base, bool bf16, uint64_t L, uint64_t heads, uint64_t batch,
             const int64_t* st) {
  const uint64_t dims[4] = {static_cast<uint64_t>(D), L, heads, batch};
  const uint64_t strides[3] = {static_cast<uint64_t>(st[0]) * 2, static_cast<uint64_t>(st[1]) * 2,
                               static_cast<uint64_t>(st[2]) * 2};
  const uint32_t box[4] = {64, 128, 1, 1};
  return make_map_16bit(tm, base, bf16, 4, dims, strides, box);
}

template <bool BF16>
int launch(const void* q, const void* k, const void* v, const int64_t* qs, const int64_t* ks,
           const int64_t* vs, const Params& p, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  const uint64_t heads = static_cast<uint64_t>(p.heads), batch = static_cast<uint64_t>(p.bh / p.heads);
  int s = make_map(&tq, q, BF16, p.L, heads, batch, qs);
  if (!s) s = make_map(&tk, k, BF16, p.L, heads, batch, ks);
  if (!s) s = make_map(&tv, v, BF16, p.L, heads, batch, vs);
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

namespace {
int sdpa_entry(const void* q, const void* k, const void* v, void* o, int64_t batch, int64_t heads, int64_t L,
               int64_t D, const int64_t* qs, const int64_t* ks, const int64_t* vs, float scale, int causal,
               int dtype, int* error_flag, void* stream) {
  PHEW_REQUIRE(q && k && v && o, "phew_sdpa: null pointer");
  PHEW_REQUIRE(phew_sdpa_supported(L, D, dtype), "phew_sdpa: needs D == 128, L % 128 == 0, bf16/f16");
  PHEW_REQUIRE(batch > 0 && heads > 0 && batch * heads * L < (1LL << 31), "phew_sdpa: bad batch");
  // The row max is taken over the unscaled scores.
  PHEW_REQUIRE(scale > 0.0f, "phew_sdpa: scale must be positive");
  PHEW_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                 reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15) == 0,
               "phew_sdpa: pointers must be 16-byte aligned");
  for (const int64_t* st : {qs, ks, vs})
    for (int i = 0; i < 3; ++i)
      PHEW_REQUIRE(st[i] > 0 && (st[i] * 2) % 16 == 0, "phew_sdpa: strides must be positive multiples of 16 bytes");
  attn::Params p;
  p.L = static_cast<int>(L);
  p.bh = static_cast<int>(batch * heads);
  p.heads = static_cast<int>(heads);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.O = o;
  p.error_flag = error_flag;
  const tc::TestStall stall = tc::take_test_stall();
  p.wait_ns = stall.wait_ns;
  p.withhold = stall.withhold;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == PHEW_BF16 ? attn::launch<true>(q, k, v, qs, ks, vs, p, st)
                            : attn::launch<false>(q, k, v, qs, ks, vs, p, st);
}
}  // namespace

extern "C" int phew_sdpa(const void* q, const void* k, const void* v, void* o, int64_t batch_heads,
                         int64_t L, int64_t D, float scale, int causal, int dtype, int* error_flag,
                         void* stream) {
  // contiguous [batch_heads, L, D]: one "head" axis of extent 1
  const int64_t st[3] = {D, L * D, L * D};
  return sdpa_entry(q, k, v, o, batch_heads, 1, L, D, st, st, st, scale, causal, dtype, error_flag, stream);
}

extern "C" int phew_sdpa_strided(const void* q, const void* k, const void* v, void* o, int64_t batch,
                                 int64_t heads, int64_t L, int64_t D, const int64_t* q_strides,
                                 const int64_t* k_strides, const int64_t* v_strides, float scale, int causal,
                                 int dtype, int* error_flag, void* stream) {
  PHEW_REQUIRE(q_strides && k_strides && v_strides, "phew_sdpa_strided: null strides");
  return sdpa_entry(q, k, v, o, batch, heads, L, D, q_strides, k_strides, v_strides, scale, causal, dtype,
                    error_flag, stream);
}
