// Dense GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   C[b, m, n] = sum_k A[b, m, k] * B[b, k, n]      (bf16 or fp16 in, fp32 accumulate)
//   optional fused row scale: C[b, m, :] *= rsqrt(mean_k(A[b, m, k]^2) + eps)
//
// Stands in for `a @ b` (phew emit/codegen.py:129-133, MatMul ir/ops.py:35-40)
// and, with the row scale, for the normed matmul `(x @ W) * rsqrt(mean(x^2) + eps)`
// that rules/primitive_subst.py:156-240 rewrites to rms_norm(x) @ W.
//
// Layout in HBM: A row-major [M, K] (K-major operand).  B either row-major
// [K, N] (N contiguous: an MN-major operand, `b_layout = 0`) or row-major
// [N, K] (K contiguous: a K-major operand, `b_layout = 1`, e.g. k.T in q @ k.T).
// Batches are strided; a zero batch stride broadcasts the operand.
//
// Tiles are (MT x 128) x BN (BN = 128 or 256, MT = 1 or 2; with MT = 2 the
// last, partial round of tiles runs as 128-row half tiles).  The kernel is
// persistent: at most one CTA per SM, each walking the tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... with ACC (1 or 2) accumulators in TMEM, so the
// epilogue of one tile overlaps the main loop of the next when ACC = 2, and
// the TMA producer runs ahead across tile boundaries either way:
//   warp 0      TMA producer: 128B-swizzled tiles of A and B into a STAGES-deep
//               shared-memory ring; each CTA loads its own tiles (these
//               kernels also run in multi-GPU jobs)
//   warp 1      allocates TMEM, one elected lane issues tcgen05.mma (M=128,
//               N=BN, K=16) into MT fp32 accumulators per tile (one per 128
//               rows, all sharing the stage's B tile) and commits each stage
//               back to the producer and each finished tile to the epilogue
//   warps 2-5   epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..), hand it back to the MMA warp after the last
//               read, scale, convert, store
// The row scale of the normed matmul comes from a short pass
// (`row_stats_kernel`: one warp per row of A, 16-byte loads, 2 bytes of HBM
// per element) that writes rsqrt(mean(A^2) + eps) per row; the GEMM is its
// programmatic dependent launch, so the GEMM's main loop overlaps the pass
// and only the epilogue waits for it (griddepcontrol.wait) before
// multiplying the fp32 accumulator by the factor.  Computing the factor
// inside the GEMM instead (from the A tiles in shared memory, or from HBM by
// the epilogue warps) was measured slower: the epilogue warps then gate the
// refill of every stage, or the next tile's main loop.
// Every mbarrier wait is bounded; a wait that runs out sets *error_flag and the
// kernel winds down instead of spinning.
#include "tc_common.cuh"

#include <mutex>
#include <string>

namespace phew {
namespace gemm {

using namespace tc;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int kNumThreads = 192;
constexpr int kGroupM = 8;  // row blocks per group of the tile order

// A CTA computes MT x 128 rows by BN columns: MT accumulators of 128 x BN in
// TMEM that share every B tile (MT = 2 halves the B bytes per MMA).
//
// BRES (resident B, for K <= BRES_KB * 64): the CTA's work is whole column
// runs (one batch entry and column block, every row block in order); the
// run's B block stays in shared memory and only A tiles stream through the
// ring.  With K = 128 the output write is the whole cost, and a tile read
// its A and B (96 KB) from the L2 for every 64 KB it wrote: the L2 carried
// 2.7 times the DRAM bytes and bound the kernel.  Resident B reads 32 KB per
// 64 KB written.
template <int BN, int MT, int ACC, bool BRES = false> struct Cfg {
  static constexpr int ROWS = BM * MT;
  static constexpr int A_BYTES = ROWS * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int BRES_KB = 2;
  static constexpr int BRES_BYTES = BRES ? BRES_KB * B_BYTES : 0;
  static constexpr int STAGE_BYTES = BRES ? A_BYTES : A_BYTES + B_BYTES;
  static constexpr int STAGES = BRES ? 6 : (200 * 1024) / STAGE_BYTES;
  // epilogue staging for TMA stores: 4 warps x 2 buffers x (32 rows x 128 B)
  static constexpr int OUT_BYTES = 4 * 2 * 32 * 128;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BRES_BYTES + OUT_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = BN * MT * ACC;
  static_assert(TMEM_COLS <= 512, "accumulators exceed TMEM");
  static_assert(!BRES || MT == 1, "resident B walks 128-row blocks");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert((2 * STAGES + 2 * ACC + 4) * 8 <= 256, "barrier area");
};

struct Params {
  int M, N, K;
  int b_mn_major;  // 1: B is [K, N] (N contiguous)
  int batch;
  // Batch entry bz of A / B is (bz / batch_inner, bz % batch_inner) of two
  // batch axes with their own strides (e.g. (batch, head) of q sliced out of
  // a fused qkv projection): the operand maps are 4-D, [K or N, rows, inner,
  // outer].  One strided batch axis: batch_inner = 1.
  int batch_inner;
  long long sa_inner, sb_inner;  // strides (elements) of the inner batch axis of A / B
  int a_batched, b_batched;
  void* C;
  long long ldc;
  long long c_batch_stride;
  int out_dtype;  // PHEW_F32 / PHEW_F16 / PHEW_BF16
  int row_scale;  // 1: rows scaled by rsqrt(mean(A^2) + eps); 2: rows replaced by sum(A^2)
  int tma_store;  // 1: 16-bit C written by TMA stores through shared memory
  float eps;
  int* error_flag;
  const float* row_vec;  // row_scale != 0: the per-row factor (or sum), [a_batched ? batch : 1][M]
  unsigned long long wait_ns;  // bound of every pipeline wait
  int withhold;                // test hook: k-block load left unissued (-1: none)
};

// Sum of squares of one row of A (K elements) by one warp: 16-byte loads,
// sixteen in flight per lane (a whole 4096-element 16-bit row per warp: the
// loop is bound by memory latency, not bandwidth, otherwise) when the row
// is 16-byte aligned, fp32 accumulation, lanes combined by a butterfly;
// every lane gets the sum.
template <typename T>
__device__ __forceinline__ float row_sumsq(const T* __restrict__ row, int K, int lane) {
  constexpr int U = 16;
  float ss = 0.f;
  int k0 = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    constexpr int E = 16 / sizeof(T);
    const int nv = K / E;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int v = lane;
    for (; v + 32 * (U - 1) < nv; v += 32 * U) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = __ldg(rv + v + 32 * u);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const float x = to_f32(e[i]);
          acc[u & 3] = fmaf(x, x, acc[u & 3]);
        }
      }
    }
    for (; v < nv; v += 32) {
      const uint4 raw = __ldg(rv + v);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const float x = to_f32(e[i]);
        acc[0] = fmaf(x, x, acc[0]);
      }
    }
    ss = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    k0 = nv * E;
  }
  for (int k = k0 + lane; k < K; k += 32) {
    const float x = to_f32(row[k]);
    ss = fmaf(x, x, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return ss;
}

__device__ __forceinline__ float row_stat_value(float ss, int K, int mode, float eps) {
  return mode == 2 ? ss : 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
}

// Per-row statistic of A for the row scale: mode 1 writes
// rsqrt(sum(A[m, :]^2) / K + eps), mode 2 the sum of squares itself.  One
// warp per row.
template <typename T>
__global__ void __launch_bounds__(256, 1) row_stats_kernel(const T* __restrict__ A, float* __restrict__ out, int M, int nb, int K,
                                 long long lda, long long sa, int mode, float eps) {
  // The GEMM that reads `out` may start now (it waits for this grid's
  // completion before its first epilogue).
  asm volatile("griddepcontrol.launch_dependents;");
  const int warps = static_cast<int>(gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(nb) * M;
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const float ss = row_sumsq(A + (r / M) * sa + (r % M) * lda, K, lane);
    if (lane == 0) out[r] = row_stat_value(ss, K, mode, eps);
  }
}

template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const float* v, int ncols) {
  if (ncols >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    constexpr int PER = 16 / sizeof(T);
#pragma unroll
    for (int c = 0; c < 32; c += PER) {
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(v[c + i]);
      *reinterpret_cast<uint4*>(dst + c) = raw;
    }
  } else {
    for (int i = 0; i < 32 && i < ncols; ++i) dst[i] = from_f32<T>(v[i]);
  }
}

// Two fp32 values rounded (to nearest even) into a packed bf16x2 / f16x2 word.
__device__ __forceinline__ uint32_t pack_out(float lo, float hi, bool bf16) {
  uint32_t d;
  if (bf16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// RS: the row-scale variant (a separate instantiation, so the plain GEMM's
// epilogue compiles without the factor read: with it in the same body the
// write-bound QK^T-shaped GEMM ran 50 % slower).
template <int BN, int MT, int ACC, bool BF16, bool RS, bool BRES>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const Params p) {
  using C = Cfg<BN, MT, ACC, BRES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_res = smem + C::STAGES * C::STAGE_BYTES;  // [BRES_KB][B tile] (BRES only)
  uint8_t* out_stage = b_res + C::BRES_BYTES;           // [4 warps][2][32 x 128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + C::OUT_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;  // [ACC]: accumulator a holds a finished tile
  uint64_t* acc_empty = acc_full + ACC;    // [ACC]: the epilogue has read accumulator a
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + ACC);
  uint64_t* drain = acc_empty + ACC + 1;   // the MMA thread's last commit (failure path)
  uint64_t* b_full = drain + 1;            // BRES: the run's B block landed
  uint64_t* b_empty = drain + 2;           // BRES: the run's last MMAs completed

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (p.K + BK - 1) / BK;
  const int n_nb = (p.N + BN - 1) / BN;
  const int n_mb = (p.M + C::ROWS - 1) / C::ROWS;
  const int num_tiles = n_nb * n_mb * p.batch;
  // Tile t -> (batch, row block, column block) in groups of kGroupM row
  // blocks: within a group the row blocks go fastest, then the column
  // blocks, so the ~148 tiles in flight cover about kGroupM row blocks by
  // 148 / kGroupM column blocks and both their A rows and their B columns
  // stay in L2 (with column blocks fastest over a wide B, every band of rows
  // streamed all of B from HBM again).
  // A GEMM with few k-blocks (q @ k^T, K = 128) is bound by writing C, not
  // by its operands: it keeps column blocks fastest, so the tiles in flight
  // write whole rows of C together.
  const int tiles_per_batch = n_nb * n_mb;
  const bool col_fastest = num_kb < 8;
  auto coords = [&](int t, int& bz, int& m0, int& n0) {
    bz = t / tiles_per_batch;
    const int tt = t - bz * tiles_per_batch;
    if (col_fastest) {
      n0 = (tt % n_nb) * BN;
      m0 = (tt / n_nb) * C::ROWS;
      return;
    }
    const int g = tt / (kGroupM * n_nb);
    const int first_m = g * kGroupM;
    const int gsize = n_mb - first_m < kGroupM ? n_mb - first_m : kGroupM;
    const int within = tt - g * kGroupM * n_nb;
    m0 = (first_m + within % gsize) * C::ROWS;
    n0 = (within / gsize) * BN;
  };
  // Wave quantization: with two 128-row halves per tile (MT = 2), the last,
  // partial round of tiles runs as twice as many 128-row half tiles when they
  // fit in one round, so that round takes half as long.  Work item w -> tile
  // coordinates and the number of 128-row halves it covers (mt); every role
  // walks the same items.
  const int rem = num_tiles % static_cast<int>(gridDim.x);
  const bool split = MT == 2 && num_tiles > static_cast<int>(gridDim.x) && rem > 0 &&
                     2 * rem <= static_cast<int>(gridDim.x);
  const int first_half = split ? num_tiles - rem : num_tiles;
  const int num_work = split ? num_tiles + rem : num_tiles;
  auto work = [&](int w, int& bz, int& m0, int& n0, int& mt) {
    if (w < first_half) {
      coords(w, bz, m0, n0);
      mt = MT;
      return;
    }
    const int u = w - first_half;
    coords(first_half + u / 2, bz, m0, n0);
    m0 += (u & 1) * BM;
    mt = 1;
  };
  // The i-th item of this CTA; false past its last.  Tiles: every
  // gridDim.x-th work item.  BRES: column runs blockIdx.x, blockIdx.x +
  // gridDim.x, ..., each its n_mb row blocks in order, so that the CTAs
  // walk the row blocks of neighbouring column blocks together and share
  // their A rows through the L2.
  const int num_runs = p.batch * n_nb;
  auto item = [&](int i, int& bz, int& m0, int& n0, int& mt) -> bool {
    if constexpr (BRES) {
      const int run = blockIdx.x + (i / n_mb) * static_cast<int>(gridDim.x);
      if (run >= num_runs) return false;
      bz = run / n_nb;
      n0 = (run - bz * n_nb) * BN;
      m0 = (i % n_mb) * BM;
      mt = 1;
      return true;
    } else {
      const int t = blockIdx.x + i * static_cast<int>(gridDim.x);
      if (t >= num_work) return false;
      work(t, bz, m0, n0, mt);
      return true;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // MMA commit
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(drain, 1);
    mbar_init(b_full, 1);
    mbar_init(b_empty, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  uint32_t kg_armed = 0;  // producer: k-blocks whose loads were issued (ring positions 0..kg_armed-1)
  uint32_t b_armed = 0;   // producer (BRES): runs whose B block load was issued

  if (warp == 0) {
    // ---------------- TMA producer: runs ahead across tiles ----------------
    if (lane == 0) {
      uint32_t kg = 0;  // k-blocks issued so far (ring position)
      for (int i = 0; ok; ++i) {
        int bz, m0, n0, mt;
        if (!item(i, bz, m0, n0, mt)) break;  // a half tile loads the full box from its own first row
        const int bi = bz % p.batch_inner, bo = bz / p.batch_inner;
        const int ba_i = p.a_batched ? bi : 0, ba_o = p.a_batched ? bo : 0;
        const int bb_i = p.b_batched ? bi : 0, bb_o = p.b_batched ? bo : 0;
        if (BRES && i % n_mb == 0) {
          // a new run: its B block replaces the last one once that run's MMAs are done
          const uint32_t rk = static_cast<uint32_t>(i / n_mb);
          if (!mbar_wait(b_empty, (rk & 1) ^ 1, p.error_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          b_armed = rk + 1;
          mbar_expect_tx(b_full, num_kb * C::B_BYTES);
          for (int kb = 0; kb < num_kb; ++kb) {
            uint8_t* sb = b_res + kb * C::B_BYTES;
            if (p.b_mn_major) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_4d(sb + j * (64 * BK * 2), &tmB, b_full, n0 + j * 64, kb * BK, bb_i, bb_o);
            } else {
              tma_load_4d(sb, &tmB, b_full, kb * BK, n0, bb_i, bb_o);
            }
          }
        }
        for (int kb = 0; kb < num_kb; ++kb, ++kg) {
          const int s = kg % C::STAGES;
          const uint32_t ph = (kg / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.error_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          kg_armed = kg + 1;
          if (static_cast<int>(kg) == p.withhold) continue;  // test hook: this stage never fills
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          mbar_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_4d(sa, &tmA, &full[s], kb * BK, m0, ba_i, ba_o);
          if (BRES) {
            // B is resident for the run
          } else if (p.b_mn_major) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_4d(sb + j * (64 * BK * 2), &tmB, &full[s], n0 + j * 64, kb * BK, bb_i, bb_o);
          } else {
            tma_load_4d(sb, &tmB, &full[s], kb * BK, n0, bb_i, bb_o);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_f16(BF16 ? 1 : 0, 0, BM, BN);
      const uint32_t idesc_b = p.b_mn_major ? instr_desc_f16(BF16 ? 1 : 0, 1, BM, BN) : idesc;
      uint32_t kg = 0, it = 0;
      for (int i = 0; ok; ++i, ++it) {
        int bz, m0, n0, mt;
        if (!item(i, bz, m0, n0, mt)) break;
        if (BRES && i % n_mb == 0) {
          // the run's B block
          if (!mbar_wait(b_full, static_cast<uint32_t>(i / n_mb) & 1, p.error_flag, p.wait_ns)) {
            ok = false;
            break;
          }
        }
        const int a = it % ACC;
        // accumulator a is free once the epilogue has read the tile before
        if (!mbar_wait(&acc_empty[a], ((it / ACC) & 1) ^ 1, p.error_flag, p.wait_ns)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + a * (MT * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++kg) {
          const int s = kg % C::STAGES;
          const uint32_t ph = (kg / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.error_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = BRES ? smem_u32(b_res + kb * C::B_BYTES) : sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = p.b_mn_major ? smem_desc(sb + kk * (16 * 128), 64 * BK * 2, 1024)
                                             : smem_desc(sb + kk * 32, 16, 1024);
#pragma unroll
            for (int h = 0; h < MT; ++h) {
              if (h >= mt) break;
              // rows h*128.. of the A tile start h*128*128 bytes in (1024-aligned)
              const uint64_t ad = smem_desc(sa + h * (BM * 128) + kk * 32, 16, 1024);
              mma_ss(acc + h * BN, ad, bd, idesc_b, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          commit(&empty[s]);
        }
        if (ok) commit(&acc_full[a]);
        // the run's last tile: its B block may be replaced once these MMAs are done
        if (ok && BRES && i % n_mb == n_mb - 1) commit(b_empty);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    // With the row scale, the factors come from row_stats_kernel, launched
    // just before this kernel as its programmatic-dependency primary: wait
    // (once, before the first epilogue reads them) for it to complete.
    bool rows_ready = !RS;
    uint32_t it = 0, out_idx = 0;
    for (int i = 0; ok; ++i, ++it) {
      int bz, m0, n0, mt;
      if (!item(i, bz, m0, n0, mt)) break;
      const int a = it % ACC;
      if (ok && !mbar_wait(&acc_full[a], (it / ACC) & 1, p.error_flag, p.wait_ns)) ok = false;
      if (!ok) break;
      if (!rows_ready) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        rows_ready = true;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem + a * (MT * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      if (p.tma_store) {
        // 64 columns at a time: TMEM -> registers -> this warp's 32 x 64
        // staging box (128B-swizzled, so the 8 lanes of a store phase hit
        // distinct banks) -> one TMA store of the box, double-buffered.
        uint8_t* my_out = out_stage + (warp - 2) * (2 * 32 * 128);
        for (int h = 0; h < mt; ++h) {
          const int srow = m0 + h * BM + quarter * 32 + lane;
          const float scale = (RS && srow < p.M) ? p.row_vec[(p.a_batched ? bz : 0) * p.M + srow] : 1.0f;
#pragma unroll 1
          for (int c = 0; c < BN; c += 64, ++out_idx) {
            uint32_t r[64];
            tmem_ld32(acc + h * BN + c, r);
            tmem_ld32(acc + h * BN + c + 32, r + 32);
            tmem_ld_wait();
            if (h == mt - 1 && c + 64 == BN) {
              // last read of this accumulator: hand it back to the MMA warp
              asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[a]);
            }
            uint8_t* box = my_out + (out_idx & 1) * (32 * 128);
            if (lane == 0) bulk_wait_read1();  // the store issued two boxes ago has read this one
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint32_t w[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float lo = __uint_as_float(r[8 * j + 2 * q]), hi = __uint_as_float(r[8 * j + 2 * q + 1]);
                if (RS) {
                  if (p.row_scale == 1) {
                    lo *= scale;
                    hi *= scale;
                  } else {  // diagnostic: the row's sum of squares
                    lo = hi = scale;
                  }
                }
                w[q] = pack_out(lo, hi, p.out_dtype == PHEW_BF16);
              }
              *reinterpret_cast<uint4*>(box + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                  make_uint4(w[0], w[1], w[2], w[3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmC, box, n0 + c, m0 + h * BM + quarter * 32, bz);
              bulk_commit();
            }
          }
        }
        continue;
      }
      for (int h = 0; h < mt; ++h) {
        const int row = m0 + h * BM + quarter * 32 + lane;
        const float scale = (RS && row < p.M) ? p.row_vec[(p.a_batched ? bz : 0) * p.M + row] : 1.0f;
        const long long cbase = static_cast<long long>(bz) * p.c_batch_stride + static_cast<long long>(row) * p.ldc;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          {
            uint32_t r[32];
            tmem_ld32(acc + h * BN + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          }
          if (h == mt - 1 && c + 32 == BN) {
            // last read of this accumulator: hand it back to the MMA warp
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
          }
          if (row < p.M && n0 + c < p.N) {
            if (RS && p.row_scale == 1) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= scale;
            } else if (RS) {  // diagnostic: the row's sum of squares
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = scale;
            }
            const int ncols = p.N - (n0 + c);
            if (p.out_dtype == PHEW_BF16)
              store_row32(static_cast<bf16*>(p.C) + cbase + n0 + c, v, ncols);
            else if (p.out_dtype == PHEW_F16)
              store_row32(static_cast<f16*>(p.C) + cbase + n0 + c, v, ncols);
            else
              store_row32(static_cast<float*>(p.C) + cbase + n0 + c, v, ncols);
          }
        }
      }
    }
    // TMA stores must finish reading shared memory before the CTA exits.
    if (lane == 0) bulk_wait_all();
  }
  if (!ok && p.error_flag) atomicExch(p.error_flag, PHEW_ERR_TIMEOUT);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (__syncthreads_or(!ok)) {
    // A wait ran out somewhere in the CTA: before the shared memory and the
    // TMEM are given back, let the work this CTA still has in flight land
    // (each wait bounded again): the tile loads of the ring positions the
    // producer armed last, and the MMAs the issuer committed.
    if (warp == 0 && lane == 0) {
      const uint32_t first = kg_armed > static_cast<uint32_t>(C::STAGES) ? kg_armed - C::STAGES : 0;
      for (uint32_t i = first; i < kg_armed; ++i) {
        if (static_cast<int>(i) == p.withhold) continue;
        mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, nullptr, p.wait_ns);
      }
      // the last B block load (a run's load is issued only after the one before was consumed)
      if (BRES && b_armed > 0) mbar_wait(b_full, (b_armed - 1) & 1, nullptr, p.wait_ns);
    } else if (warp == 1 && lane == 0) {
      commit(drain);
      mbar_wait(drain, 0, nullptr, p.wait_ns);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// SIMT fallback for shapes the TMA path cannot describe (row strides that are
// not multiples of 16 bytes): 16 x 16 output tiles, fp32 accumulation.
template <typename T>
__global__ void gemm_simt_kernel(const T* A, const T* B, Params p, long long lda, long long ldb,
                                 long long sa, long long sb, long long sa_in, long long sb_in) {
  __shared__ float ta[16][17];
  __shared__ float tb[16][17];
  const int bz = blockIdx.z;
  const int bi = bz % p.batch_inner, bo = bz / p.batch_inner;
  const int row = blockIdx.y * 16 + threadIdx.y;
  const int col = blockIdx.x * 16 + threadIdx.x;
  const T* Ab = A + (p.a_batched ? bo * sa + bi * sa_in : 0);
  const T* Bb = B + (p.b_batched ? bo * sb + bi * sb_in : 0);
  float acc = 0.f;
  for (int k0 = 0; k0 < p.K; k0 += 16) {
    const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    ta[threadIdx.y][threadIdx.x] = (row < p.M && ka < p.K) ? to_f32(Ab[row * lda + ka]) : 0.f;
    float bv = 0.f;
    if (col < p.N && kb < p.K)
      bv = p.b_mn_major ? to_f32(Bb[static_cast<long long>(kb) * ldb + col])
                        : to_f32(Bb[static_cast<long long>(col) * ldb + kb]);
    tb[threadIdx.y][threadIdx.x] = bv;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(ta[threadIdx.y][k], tb[k][threadIdx.x], acc);
    __syncthreads();
  }
  if (row < p.M && col < p.N) {
    const float rv = p.row_scale ? p.row_vec[(p.a_batched ? bz : 0) * p.M + row] : 1.f;
    const long long o = static_cast<long long>(bz) * p.c_batch_stride + static_cast<long long>(row) * p.ldc + col;
    const float v = p.row_scale == 2 ? rv : acc * rv;
    if (p.out_dtype == PHEW_BF16) static_cast<bf16*>(p.C)[o] = from_f32<bf16>(v);
    else if (p.out_dtype == PHEW_F16) static_cast<f16*>(p.C)[o] = from_f32<f16>(v);
    else static_cast<float*>(p.C)[o] = v;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int make_map(CUtensorMap* tm, const void* base, bool bf16, uint64_t d0, uint64_t d1, uint64_t d2,
             uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0, uint32_t b1) {
  const uint64_t dims[3] = {d0, d1, d2};
  const uint64_t strides[2] = {s1_bytes, s2_bytes};
  const uint32_t box[3] = {b0, b1, 1};
  return make_map_16bit(tm, base, bf16, 3, dims, strides, box);
}

// An operand [outer][inner][rows][cols] of 16-bit elements: cols contiguous,
// rows `ld` apart, the two batch axes their own strides (elements).
int make_operand_map(CUtensorMap* tm, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                     uint64_t inner, uint64_t outer, long long ld, long long s_inner, long long s_outer,
                     uint32_t b0, uint32_t b1) {
  const uint64_t dims[4] = {cols, rows, inner, outer};
  const uint64_t strides[3] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(s_inner) * 2,
                               static_cast<uint64_t>(s_outer) * 2};
  const uint32_t box[4] = {b0, b1, 1, 1};
  return make_map_16bit(tm, base, bf16, 4, dims, strides, box);
}

// A memory pool per device for the row factors that keeps what it has
// reserved (the default pool returns memory at every synchronisation and
// maps it again on the next call).
cudaMemPool_t row_pool() {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) return nullptr;
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = pool;
  }
  return pools[dev];
}

template <typename T>
int launch_row_stats(const void* A, float* out, const Params& p, long long lda, long long sa, cudaStream_t st) {
  // Keep the SM's shared memory configured for the GEMM CTA that starts
  // beside this kernel (a small carveout would hold the GEMM back until
  // these blocks leave).
  static bool carveout = false;
  if (!carveout) {
    PHEW_CHECK_CUDA(cudaFuncSetAttribute(row_stats_kernel<T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         static_cast<int>(cudaSharedmemCarveoutMaxShared)));
    carveout = true;
  }
  const int nb = p.a_batched ? p.batch : 1;
  const long long rows = static_cast<long long>(nb) * p.M;
  // One 256-thread block per SM: 8 warps x a whole row each in flight
  // saturate HBM, and the SM keeps room for the GEMM CTA that starts beside
  // it (programmatic dependent launch).
  long long blocks = (rows + 7) / 8;
  const long long cap = static_cast<long long>(sm_count_current());
  if (blocks > cap) blocks = cap;
  row_stats_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(static_cast<const T*>(A), out, p.M, nb, p.K,
                                                                     lda, sa, p.row_scale, p.eps);
  return launch_status("row_stats_kernel");
}

// Persistent grid: one CTA per SM at most, each looping over tiles.
int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

template <int BN, int MT, int ACC, bool BF16>
int launch_tc(const void* A, const void* B, const Params& p, long long lda, long long ldb,
              long long sa, long long sb, cudaStream_t st) {
  using C = Cfg<BN, MT, ACC>;
  CUtensorMap ta, tb;
  // [outer][inner][rows][cols] views; an axis of extent 1 gets the stride of
  // the whole matrix (any multiple of 16 bytes describes it)
  const uint64_t bi = static_cast<uint64_t>(p.batch_inner), bo = static_cast<uint64_t>(p.batch / p.batch_inner);
  const long long a_mat = static_cast<long long>(p.M) * lda;
  const long long b_mat = static_cast<long long>(p.b_mn_major ? p.K : p.N) * ldb;
  const bool a_in = p.a_batched && bi > 1, b_in = p.b_batched && bi > 1;
  int s = make_operand_map(&ta, A, BF16, p.K, p.M, a_in ? bi : 1, p.a_batched ? bo : 1, lda,
                           a_in ? p.sa_inner : a_mat, p.a_batched ? sa : a_mat, BK, C::ROWS);
  if (s) return s;
  if (p.b_mn_major)
    s = make_operand_map(&tb, B, BF16, p.N, p.K, b_in ? bi : 1, p.b_batched ? bo : 1, ldb,
                         b_in ? p.sb_inner : b_mat, p.b_batched ? sb : b_mat, 64, BK);
  else
    s = make_operand_map(&tb, B, BF16, p.K, p.N, b_in ? bi : 1, p.b_batched ? bo : 1, ldb,
                         b_in ? p.sb_inner : b_mat, p.b_batched ? sb : b_mat, BK, BN);
  if (s) return s;
  // C through TMA stores when it is 16-bit and its layout is describable
  // (16-byte aligned base and row/batch strides); otherwise direct stores.
  CUtensorMap tc;
  Params q = p;
  const long long cbs = p.batch > 1 ? p.c_batch_stride : static_cast<long long>(p.M) * p.ldc;
  q.tma_store = p.out_dtype != PHEW_F32 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0 &&
                (p.ldc * 2) % 16 == 0 && (cbs * 2) % 16 == 0 && cbs > 0 && p.ldc >= p.N;
  if (q.tma_store &&
      make_map(&tc, p.C, p.out_dtype == PHEW_BF16, p.N, p.M, p.batch, p.ldc * 2, cbs * 2, 64, 32) != PHEW_OK)
    q.tma_store = 0;
  if (!q.tma_store) tc = ta;  // unused
  if constexpr (MT == 1) {
    // K <= 128, enough row blocks per run to amortise loading B once, and
    // enough runs to keep every SM busy: resident B, one CTA per column run
    // at a time
    const int num_kb = (p.K + BK - 1) / BK;
    const long long n_mb = (p.M + BM - 1) / BM;
    const long long n_runs = static_cast<long long>((p.N + BN - 1) / BN) * p.batch;
    using CR = Cfg<BN, MT, ACC, true>;
    if (!q.row_scale && num_kb <= CR::BRES_KB && n_mb >= 8 && n_runs >= 2LL * sm_count() &&
        n_runs * n_mb < (1LL << 31)) {
      static bool attr_res = false;
      if (!attr_res) {
        PHEW_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, MT, ACC, BF16, false, true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, CR::SMEM));
        attr_res = true;
      }
      const unsigned grid = static_cast<unsigned>(sm_count());
      gemm_tc_kernel<BN, MT, ACC, BF16, false, true><<<grid, kNumThreads, CR::SMEM, st>>>(ta, tb, tc, q);
      return launch_status("gemm_tc_kernel");
    }
  }
  static bool attr_set = false;
  if (!attr_set) {
    PHEW_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, MT, ACC, BF16, false, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    PHEW_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, MT, ACC, BF16, true, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set = true;
  }
  const long long tiles = static_cast<long long>((p.N + BN - 1) / BN) * ((p.M + C::ROWS - 1) / C::ROWS) * p.batch;
  PHEW_REQUIRE(tiles < (1LL << 31), "phew_gemm: too many tiles");
  const unsigned grid = static_cast<unsigned>(tiles < sm_count() ? tiles : sm_count());
  if (q.row_scale) {
    // Programmatic dependent launch after row_stats_kernel: the main loop
    // overlaps that pass; the epilogue waits for it (griddepcontrol.wait).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kNumThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PHEW_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, MT, ACC, BF16, true, false>, ta, tb, tc, q));
    return launch_status("gemm_tc_kernel");
  }
  gemm_tc_kernel<BN, MT, ACC, BF16, false, false><<<grid, kNumThreads, C::SMEM, st>>>(ta, tb, tc, q);
  return launch_status("gemm_tc_kernel");
}

int gemm_dispatch(const void* A, const void* B, const Params& p, int64_t lda, int64_t ldb, int64_t stride_a,
                  int64_t stride_b, int in_dtype, cudaStream_t st);

// The tensor-core kernels take 16-bit operands whose bases and row / batch
// strides are 16-byte aligned (TMA); anything else goes to the SIMT kernel.
inline bool uses_tensor_cores(const void* A, const void* B, int64_t lda, int64_t ldb, int64_t stride_a,
                              int64_t stride_b, int64_t K, int in_dtype, int64_t sa_inner = 0,
                              int64_t sb_inner = 0) {
  return in_dtype != PHEW_F32 && K > 0 &&
         ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) == 0 && (lda * 2) % 16 == 0 &&
         (ldb * 2) % 16 == 0 && (stride_a * 2) % 16 == 0 && (stride_b * 2) % 16 == 0 &&
         (sa_inner * 2) % 16 == 0 && (sb_inner * 2) % 16 == 0;
}

}  // namespace gemm
}  // namespace phew

using namespace phew;
using namespace phew::gemm;

namespace {
int gemm_entry(const void* A, const void* B, void* Cout, int64_t M, int64_t N, int64_t K, int64_t batch,
               int64_t batch_inner, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a, int64_t stride_a_inner,
               int64_t stride_b, int64_t stride_b_inner, int64_t stride_c, int b_layout, int in_dtype,
               int out_dtype, int row_scale, float eps, int* error_flag, void* stream) {
  PHEW_REQUIRE(A && B && Cout, "phew_gemm: null operand");
  PHEW_REQUIRE(M >= 0 && N >= 0 && K >= 0 && batch >= 1, "phew_gemm: bad shape");
  PHEW_REQUIRE(batch_inner >= 1 && batch % batch_inner == 0, "phew_gemm: batch_inner must divide batch");
  PHEW_REQUIRE(batch_inner == 1 || row_scale == 0, "phew_gemm: the row scale takes one batch axis");
  PHEW_REQUIRE(batch_inner == 1 || ((stride_a == 0) == (stride_a_inner == 0) && (stride_b == 0) == (stride_b_inner == 0)),
               "phew_gemm: an operand is batched over both batch axes or over neither");
  PHEW_REQUIRE(in_dtype == PHEW_BF16 || in_dtype == PHEW_F16 || in_dtype == PHEW_F32,
               "phew_gemm: bad input dtype");
  PHEW_REQUIRE(out_dtype == PHEW_BF16 || out_dtype == PHEW_F16 || out_dtype == PHEW_F32,
               "phew_gemm: bad output dtype");
  PHEW_REQUIRE(b_layout == 0 || b_layout == 1, "phew_gemm: b_layout must be 0 ([K,N]) or 1 ([N,K])");
  PHEW_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && batch < 65536,
               "phew_gemm: extent too large");
  if (M == 0 || N == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.b_mn_major = b_layout == 0 ? 1 : 0;
  p.batch = static_cast<int>(batch);
  p.batch_inner = static_cast<int>(batch_inner);
  p.sa_inner = stride_a_inner;
  p.sb_inner = stride_b_inner;
  p.a_batched = stride_a != 0;
  p.b_batched = stride_b != 0;
  p.C = Cout;
  p.ldc = ldc;
  p.c_batch_stride = stride_c;
  p.out_dtype = out_dtype;
  p.row_scale = row_scale;
  p.tma_store = 0;
  p.eps = eps;
  p.error_flag = error_flag;
  p.row_vec = nullptr;
  const phew::tc::TestStall stall = phew::tc::take_test_stall();
  p.wait_ns = stall.wait_ns;
  p.withhold = stall.withhold;
  if (row_scale) {
    // The per-row factor lives in stream-ordered memory allocated here and
    // freed after the GEMM on the same stream: no sharing between streams,
    // and graph capture records it as allocation / free nodes.
    PHEW_REQUIRE(row_scale == 1 || row_scale == 2, "phew_gemm: row_scale must be 0, 1 or 2");
    PHEW_REQUIRE(K > 0, "phew_gemm: the row scale needs K > 0");
    float* w = nullptr;
    const size_t bytes = static_cast<size_t>(stride_a != 0 ? batch : 1) * static_cast<size_t>(M) * sizeof(float);
    cudaMemPool_t pool = row_pool();
    PHEW_REQUIRE(pool != nullptr, "phew_gemm: no memory pool for the row factors");
    PHEW_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&w), bytes, pool, st));
    p.row_vec = w;
    int r = in_dtype == PHEW_BF16 ? launch_row_stats<bf16>(A, w, p, lda, stride_a, st)
            : in_dtype == PHEW_F16 ? launch_row_stats<f16>(A, w, p, lda, stride_a, st)
                                   : launch_row_stats<float>(A, w, p, lda, stride_a, st);
    if (!r) r = gemm_dispatch(A, B, p, lda, ldb, stride_a, stride_b, in_dtype, st);
    const cudaError_t fe = cudaFreeAsync(w, st);
    if (!r && fe != cudaSuccess) r = set_error(PHEW_ERR_CUDA, std::string("phew_gemm: cudaFreeAsync: ") + cudaGetErrorString(fe));
    return r;
  }
  return gemm_dispatch(A, B, p, lda, ldb, stride_a, stride_b, in_dtype, st);
}
}  // namespace

extern "C" int phew_gemm(const void* A, const void* B, void* Cout, int64_t M, int64_t N, int64_t K,
                         int64_t batch, int64_t lda, int64_t ldb, int64_t ldc, int64_t stride_a,
                         int64_t stride_b, int64_t stride_c, int b_layout, int in_dtype,
                         int out_dtype, int row_scale, float eps, int* error_flag, void* stream) {
  return gemm_entry(A, B, Cout, M, N, K, batch, 1, lda, ldb, ldc, stride_a, 0, stride_b, 0, stride_c, b_layout,
                    in_dtype, out_dtype, row_scale, eps, error_flag, stream);
}

extern "C" int phew_gemm_batched2(const void* A, const void* B, void* Cout, int64_t M, int64_t N, int64_t K,
                                  int64_t batch_outer, int64_t batch_inner, int64_t lda, int64_t ldb,
                                  int64_t ldc, int64_t stride_a_outer, int64_t stride_a_inner,
                                  int64_t stride_b_outer, int64_t stride_b_inner, int64_t stride_c,
                                  int b_layout, int in_dtype, int out_dtype, int* error_flag, void* stream) {
  PHEW_REQUIRE(batch_outer >= 1 && batch_inner >= 1 && batch_outer * batch_inner < 65536,
               "phew_gemm_batched2: bad batch extents");
  return gemm_entry(A, B, Cout, M, N, K, batch_outer * batch_inner, batch_inner, lda, ldb, ldc, stride_a_outer,
                    stride_a_inner, stride_b_outer, stride_b_inner, stride_c, b_layout, in_dtype, out_dtype, 0,
                    1e-5f, error_flag, stream);
}

namespace phew {
namespace gemm {

// Kernel choice for the validated call.
int gemm_dispatch(const void* A, const void* B, const Params& p, int64_t lda, int64_t ldb, int64_t stride_a,
                  int64_t stride_b, int in_dtype, cudaStream_t st) {
  const int64_t K = p.K, M = p.M, N = p.N, batch = p.batch;
  if (uses_tensor_cores(A, B, lda, ldb, stride_a, stride_b, K, in_dtype, p.sa_inner, p.sb_inner)) {
    const bool bf = in_dtype == PHEW_BF16;
    // Tile choice (every kernel is persistent: one CTA per SM looping over
    // tiles, TMA running ahead across tile boundaries):
    //   N <= 128         128 x 128 tiles, two accumulators (the epilogue of
    //                    one tile overlaps the main loop of the next)
    //   K <= 512         128 x 256, two accumulators: short main loops, so
    //                    the output write is the cost and must overlap
    //   M > 128          256 x 256 (two 128-row accumulators sharing each B
    //                    tile: 64 operand bytes per MMA cycle instead of 96)
    //   otherwise        128 x 256, two accumulators
    const bool d = bf;
    if (N <= 128) return d ? launch_tc<128, 1, 2, true>(A, B, p, lda, ldb, stride_a, stride_b, st)
                           : launch_tc<128, 1, 2, false>(A, B, p, lda, ldb, stride_a, stride_b, st);
    if (K > 512 && M > 128) return d ? launch_tc<256, 2, 1, true>(A, B, p, lda, ldb, stride_a, stride_b, st)
                                     : launch_tc<256, 2, 1, false>(A, B, p, lda, ldb, stride_a, stride_b, st);
    return d ? launch_tc<256, 1, 2, true>(A, B, p, lda, ldb, stride_a, stride_b, st)
             : launch_tc<256, 1, 2, false>(A, B, p, lda, ldb, stride_a, stride_b, st);
  }
  dim3 grid(static_cast<unsigned>((N + 15) / 16), static_cast<unsigned>((M + 15) / 16),
            static_cast<unsigned>(batch));
  dim3 block(16, 16);
  if (in_dtype == PHEW_F32)
    gemm_simt_kernel<float><<<grid, block, 0, st>>>(static_cast<const float*>(A),
                                                    static_cast<const float*>(B), p, lda, ldb,
                                                    stride_a, stride_b, p.sa_inner, p.sb_inner);
  else if (in_dtype == PHEW_BF16)
    gemm_simt_kernel<bf16><<<grid, block, 0, st>>>(static_cast<const bf16*>(A),
                                                   static_cast<const bf16*>(B), p, lda, ldb,
                                                   stride_a, stride_b, p.sa_inner, p.sb_inner);
  else
    gemm_simt_kernel<f16><<<grid, block, 0, st>>>(static_cast<const f16*>(A),
                                                  static_cast<const f16*>(B), p, lda, ldb,
                                                  stride_a, stride_b, p.sa_inner, p.sb_inner);
  return launch_status("gemm_simt_kernel");
}

}  // namespace gemm
}  // namespace phew
