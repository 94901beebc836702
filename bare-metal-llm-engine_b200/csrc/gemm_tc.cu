// gemm_tc.cu -- FP16 / BF16 GEMM on the 5th-generation tensor cores (tcgen05).
//
//   C[M,N] = A[M,K] * op(B) (+ residual),   FP32 accumulation in TMEM,
//   op(B) = B[K,N] (row-major, "MN-major" UMMA operand; the legacy matmul layout)
//        or W[N,K]^T (K-major operand; the activation x weight projection layout).
//
// One CTA per SM (persistent over output tiles), 192 threads in three roles:
//   warp 0      one elected thread issues TMA tiled loads (128-byte swizzle, no
//               multicast) of a 128x64 A tile and a BNx64 B tile per stage into a
//               multi-stage shared-memory ring guarded by full/empty mbarriers;
//   warp 1      allocates TMEM (2 accumulators x BN fp32 columns) and one thread
//               issues tcgen05.mma (M=128, N=BN, K=16, four per 64-wide k-block),
//               committing each stage back to the producer and each finished
//               accumulator to the epilogue;
//   warps 2..5  read the accumulator with tcgen05.ld (warp w owns TMEM lanes
//               32*(w%4)..+31, i.e. tile rows), add the residual in FP32, round
//               once to the 16-bit type and store -- while the MMA warp already
//               accumulates the next tile into the other TMEM buffer.
//
// Two further modes serve the small-batch projections (the HBM-bound decode
// configurations) without a second kernel:
//   SWAP  the weight W[N,K] is the UMMA "A" operand (128 weight rows per tile)
//         and the few activation rows are the "B" operand (N = 16..64), so a
//         batch of 16 still uses a full-height MMA; the epilogue writes the
//         transposed tile back into Y[M,N] (lanes = consecutive n: coalesced);
//   SPLIT the K range of each tile is divided over S CTAs of one thread-block
//         cluster (S <= 8) so that 48 weight tiles still cover all SMs; each CTA
//         parks its FP32 partial in shared memory and the partials are summed
//         in fixed rank order through distributed shared memory.
//   HILO  (with SWAP) the activation operand holds each row twice -- its FP16
//         rounding and the FP16 rounding of the remainder -- and the epilogue
//         adds the two accumulator columns, so an FP32 activation (the fused
//         RMSNorm output) is multiplied at ~FP32 accuracy.
//
// Every mbarrier wait is bounded (ENGINE_WAIT_TIMEOUT_MS, default 2 s): on expiry
// the thread sets the device error word, abandons its loop and proceeds to the
// common teardown, where TMEM is released.
#include <cooperative_groups.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace b200 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 x 16-bit = 128 bytes: one 128B-swizzle row
constexpr int kThreads = 192;
constexpr int kEpiStageBytes = 128 * 64 * 2;  // one 128-row x 64-column 16-bit tile

struct TcParams {
  int64_t K;
  int64_t num_kb;        // ceil(K / 64)
  int64_t kb_per_split;  // k-blocks per cluster rank
  int tiles_m, tiles_n;  // tile grid over (A rows, B rows)
  int split;             // S: CTAs per cluster along K (1 = no split)
  void* out;
  const void* resid;
  int64_t ldo;           // row pitch (elements) of out and resid
  int64_t out_rows;      // M of Y / C
  int64_t out_cols;      // N of Y / C
  int half_b;            // HILO: columns [half_b, 2*half_b) hold the remainders
  int vec_out;           // 16-byte output stores allowed
  int tma_epi;           // output written by TMA stores through shared memory
  unsigned int* err;
  unsigned long long limit_ns;
  // Stream-K schedule of the 2-SM kernel (sk_iters == 0: whole tiles only).
  int64_t dp_tiles;             // tiles handed out whole, round-robin over CTA pairs
  int64_t sk_iters;             // k-blocks of the remaining tiles, split evenly over pairs
  float* ws;                    // FP32 partial-tile slots: [pair][2][rank][128 x BN]
  unsigned long long* ws_cnt;   // arrival counters, zero between launches
#ifdef ENGINE_TC_TRACE
  unsigned long long* trace;  // debug builds: 8 timestamps per CTA
#endif
};

#ifdef ENGINE_TC_TRACE
#define TC_TRACE(slot)                                                                \
  do {                                                                                \
    if (p.trace) {                                                                    \
      const uint32_t cta = blockIdx.x + gridDim.x * blockIdx.z;                        \
      p.trace[cta * 8 + (slot)] = globaltimer();                                      \
    }                                                                                 \
  } while (0)
#else
#define TC_TRACE(slot) \
  do {                 \
  } while (0)
#endif

constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// SWAP (small-batch) tiles stream weights from HBM: their stage ring is kept under
// ~113 KB so two CTAs fit per SM, which lets every split-K cluster of a launch be
// resident at once (with one 190 KB CTA per SM, clusters of 3 leave SMs idle in
// each GPC and spill into a second wave).
template <int BN, bool SWAP = false>
struct TcCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages =
      SWAP ? (BN >= 64 ? 4 : (BN >= 32 ? 5 : 6))
           : ((BN >= 256) ? 4 : (BN >= 128 ? 6 : (BN >= 64 ? 8 : 10)));
  // Non-SWAP: two accumulators (double buffer across tiles).  SWAP (one tile per
  // CTA): four accumulators that take k-blocks round-robin, so four independent
  // MMA chains are in flight instead of one serial N=16..64 chain.
  static constexpr int kAccs = SWAP ? 4 : 2;
  static constexpr int kTmemCols = pow2_at_least(kAccs * BN);
  static constexpr int kPartialPitch = BN + 4;  // floats per row of the split-K partial
  static constexpr int kBarrierBytes = 256;
  static constexpr int kEpiBytes = SWAP ? 0 : 2 * kEpiStageBytes;  // TMA-store staging
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + kBarrierBytes + 1024;
  static_assert(kStages * kStageBytes >= kBM * kPartialPitch * 4, "partial must fit");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool BF16>
__device__ __forceinline__ float load16(const void* p, int64_t i) {
  if constexpr (BF16) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  } else {
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  }
}

template <bool BF16>
__device__ __forceinline__ void store16(void* p, int64_t i, float v) {
  if constexpr (BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

// Tile-order group: tiles are walked G row-tiles at a time so B tiles are reused
// from L2.  A compile-time tunable (the default is the measured best).
#ifndef ENGINE_TC_GROUP
#define ENGINE_TC_GROUP 8
#endif
// 2-SM kernel: shared-memory stages (0 = the default for the tile width).
#ifndef ENGINE_TC2_STAGES
#define ENGINE_TC2_STAGES 0
#endif

__device__ __forceinline__ void tile_coords(int64_t t, int tiles_m, int tiles_n, int& tm,
                                            int& tn) {
  constexpr int G = ENGINE_TC_GROUP;
  const int64_t per_group = static_cast<int64_t>(G) * tiles_n;
  const int64_t group = t / per_group;
  const int first_m = static_cast<int>(group * G);
  const int gsize = (tiles_m - first_m < G) ? tiles_m - first_m : G;
  const int64_t r = t % per_group;
  tm = first_m + static_cast<int>(r % gsize);
  tn = static_cast<int>(r / gsize);
}

// ---------------------------------------------------------------- stream-K
// The 2-SM kernel's work list for CTA pair q: first the whole tiles
// q, q + P, ... below dp_tiles (P = pairs in the grid), then the k-block range
// [b(q), b(q+1)), b(q) = q * sk_iters / P, of the stream-K region -- the last
// sk_iters / num_kb tiles laid end to end along K.  The host keeps that region
// between P and 2P tiles, so every range spans num_kb..2*num_kb k-blocks, has at
// most three segments, and no tile is shared by more than two pairs.  A segment
// that covers a whole tile is stored like a round-robin tile.  A partial
// segment parks its FP32 accumulator in a workspace slot and arrives on the
// tile's counter; the second arriver adds the two partials in pair order (so
// the sum does not depend on which pair finishes first) and stores the tile.
// Nothing waits on another CTA.
struct TcWork {
  int64_t tile;     // linear tile index (tile_coords order)
  int64_t kb0, kb1; // k-block range of this segment
  int64_t sk_tile;  // -1: whole tile; else tile index within the stream-K region
};

__device__ __forceinline__ int64_t sk_bound(const TcParams& p, int64_t q, int64_t npairs) {
  return q * p.sk_iters / npairs;
}

/// The pair whose range holds stream-K k-block `i` (largest q with b(q) <= i).
__device__ __forceinline__ int64_t sk_owner(const TcParams& p, int64_t i, int64_t npairs) {
  int64_t q = i * npairs / p.sk_iters;  // b(q) <= i already; step up past equal bounds
  while (q + 1 < npairs && sk_bound(p, q + 1, npairs) <= i) ++q;
  return q;
}

struct TcSched {
  int64_t t, it, it_end;
  __device__ TcSched(const TcParams& p, int64_t pair, int64_t npairs) : t(pair) {
    it = p.sk_iters > 0 ? sk_bound(p, pair, npairs) : 0;
    it_end = p.sk_iters > 0 ? sk_bound(p, pair + 1, npairs) : 0;
  }
  __device__ bool next(const TcParams& p, int64_t npairs, TcWork& w) {
    if (t < p.dp_tiles) {
      w.tile = t;
      w.kb0 = 0;
      w.kb1 = p.num_kb;
      w.sk_tile = -1;
      t += npairs;
      return true;
    }
    if (it >= it_end) return false;
    const int64_t tl = it / p.num_kb;
    const int64_t end = it_end - tl * p.num_kb;
    w.tile = p.dp_tiles + tl;
    w.kb0 = it - tl * p.num_kb;
    w.kb1 = end < p.num_kb ? end : p.num_kb;
    w.sk_tile = (w.kb0 == 0 && w.kb1 == p.num_kb) ? -1 : tl;
    it = tl * p.num_kb + w.kb1;
    return true;
  }
};

/// One CTA's partial slot: 128 rows x BN FP32 columns, stored as float4 units
/// [BN/4 column quads][128 rows] so that the 32 lanes of a warp (32 consecutive
/// rows) move 512 contiguous bytes per access.
template <int BN>
__device__ __forceinline__ float* sk_slot(const TcParams& p, int64_t pair, int slot,
                                          uint32_t rank) {
  return p.ws + ((pair * 2 + slot) * 2 + rank) * static_cast<int64_t>(128 * BN);
}

/// Partial slot (0: first segment of the pair's range, 1: last) that pair q used
/// for stream-K tile tl.
__device__ __forceinline__ int sk_slot_of(const TcParams& p, int64_t q, int64_t tl,
                                          int64_t npairs) {
  return (sk_bound(p, q, npairs) / p.num_kb == tl) ? 0 : 1;
}

/// Counts this CTA's arrival on a stream-K tile counter; returns the arrival
/// number (1-based).  acq_rel: releases this CTA's parked partial and acquires
/// the earlier arrivals'.  The CTA that stores the tile resets the counter to
/// zero, so every completed launch leaves all counters at zero (CUDA graphs
/// replay exactly); after a device-side time-out engine_device_status() zeroes
/// them again.
__device__ __forceinline__ uint32_t sk_arrive(unsigned long long* cnt) {
  unsigned long long old;
  asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(cnt) : "memory");
  return static_cast<uint32_t>(old) + 1u;
}

__device__ __forceinline__ void sk_reset(unsigned long long* cnt) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(cnt), "l"(0ull) : "memory");
}

/// Address of columns 4q..4q+3 of row rl in a partial slot.
__device__ __forceinline__ float4* sk_quad(float* slot, int quad, int rl) {
  return reinterpret_cast<float4*>(slot) + quad * 128 + rl;
}

/// Loads columns c..c+31 of row rl of the other pair's parked partial.
__device__ __forceinline__ void sk_load32(float4 x[8], const float* other, int c, int rl) {
  const float4* o = reinterpret_cast<const float4*>(other) + (c >> 2) * 128 + rl;
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = __ldcg(o + j * 128);
}

/// Adds the other pair's partial (x, from sk_load32) to 32 accumulator values
/// of this CTA (still in TMEM).  With two contributors the sum is one IEEE
/// addition, which is commutative: the result does not depend on which pair
/// arrived last.
__device__ __forceinline__ void sk_add32(uint32_t v[32], const float4 x[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j * 4 + 0] = __float_as_uint(__uint_as_float(v[j * 4 + 0]) + x[j].x);
    v[j * 4 + 1] = __float_as_uint(__uint_as_float(v[j * 4 + 1]) + x[j].y);
    v[j * 4 + 2] = __float_as_uint(__uint_as_float(v[j * 4 + 2]) + x[j].z);
    v[j * 4 + 3] = __float_as_uint(__uint_as_float(v[j * 4 + 3]) + x[j].w);
  }
}

/// Writes one output element of the tile: (rl, j) = (tile row, tile column).
template <bool SWAP, bool RESID, bool BF16>
__device__ __forceinline__ void emit(const TcParams& p, int tm, int tn, int rl, int j, int bn,
                                     float v) {
  int64_t r, c;
  if constexpr (SWAP) {
    c = static_cast<int64_t>(tm) * kBM + rl;  // weight row -> output column
    r = static_cast<int64_t>(tn) * bn + j;    // activation row -> output row
  } else {
    r = static_cast<int64_t>(tm) * kBM + rl;
    c = static_cast<int64_t>(tn) * bn + j;
  }
  if (r >= p.out_rows || c >= p.out_cols) return;
  const int64_t idx = r * p.ldo + c;
  if constexpr (RESID) v = v + load16<BF16>(p.resid, idx);
  store16<BF16>(p.out, idx, v);
}

/// Epilogue through shared memory: the four epilogue warps (128 threads, one
/// tile row each) convert 64 accumulator columns at a time into a 128-byte-
/// swizzled 16 KB staging tile (conflict-free 16-byte writes), then one thread
/// stores the tile with a TMA bulk-tensor store.  Two staging tiles alternate;
/// `chunk` counts staged chunks across tiles.  TMA clips rows / columns
/// outside the output, so edge tiles need no special case.  `other` (non-null:
/// stream-K fix-up) is the other pair's parked partial of this tile.
/// Converts 64 accumulator columns (v) into the swizzled staging tile `buf` and
/// has the elected thread store it.
template <bool BF16>
__device__ __forceinline__ void epilogue_stage_store(const CUtensorMap* tmC, uint8_t* buf,
                                                     const uint32_t (&v)[2][32], int rl,
                                                     bool elect, int32_t col, int32_t row0) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t* w = &v[j >> 2][(j & 3) * 8];
    uint4 o;
    o.x = pack2<BF16>(__uint_as_float(w[0]), __uint_as_float(w[1]));
    o.y = pack2<BF16>(__uint_as_float(w[2]), __uint_as_float(w[3]));
    o.z = pack2<BF16>(__uint_as_float(w[4]), __uint_as_float(w[5]));
    o.w = pack2<BF16>(__uint_as_float(w[6]), __uint_as_float(w[7]));
    *reinterpret_cast<uint4*>(buf + rl * 128 + ((j ^ (rl & 7)) << 4)) = o;
  }
  fence_proxy_async_smem();
  named_barrier_sync(1, 128);
  if (elect) {
    tma_store_2d(tmC, buf, col, row0);
    bulk_commit_group();
  }
}

/// Stream-K fix-up form of epilogue_tma_tile: adds the other pair's parked
/// partial of the tile.  The partial's loads run one 64-column chunk ahead of
/// the conversion, so two chunks (32 KB per warp group) are in flight.
template <int BN, bool BF16>
__device__ __forceinline__ void epilogue_tma_tile_fix(const CUtensorMap* tmC, uint8_t* stage,
                                                      uint32_t taddr, int rl, bool elect,
                                                      int32_t col_base, int32_t row0,
                                                      uint32_t& chunk, const float* other) {
  float4 x[2][2][8];
  sk_load32(x[0][0], other, 0, rl);
  sk_load32(x[0][1], other, 32, rl);
#pragma unroll
  for (int c = 0; c < BN; c += 64, ++chunk) {
    const int cur = (c >> 6) & 1;
    if (c + 64 < BN) {
      sk_load32(x[cur ^ 1][0], other, c + 64, rl);
      sk_load32(x[cur ^ 1][1], other, c + 96, rl);
    }
    uint8_t* buf = stage + (chunk & 1u) * kEpiStageBytes;
    if (elect) bulk_wait_group_read<1>();
    named_barrier_sync(1, 128);
    uint32_t v[2][32];
    tmem_ld_32x32b_x32(taddr + c, v[0]);
    tmem_ld_32x32b_x32(taddr + c + 32, v[1]);
    tmem_wait_ld();
    sk_add32(v[0], x[cur][0]);
    sk_add32(v[1], x[cur][1]);
    epilogue_stage_store<BF16>(tmC, buf, v, rl, elect, col_base + c, row0);
  }
}

template <int BN, bool BF16>
__device__ __forceinline__ void epilogue_tma_tile(const CUtensorMap* tmC, uint8_t* stage,
                                                  uint32_t taddr, int rl, bool elect,
                                                  int32_t col_base, int32_t row0,
                                                  uint32_t& chunk,
                                                  const float* other = nullptr) {
  if (other != nullptr) {
    epilogue_tma_tile_fix<BN, BF16>(tmC, stage, taddr, rl, elect, col_base, row0, chunk, other);
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN; c += 64, ++chunk) {
    uint8_t* buf = stage + (chunk & 1u) * kEpiStageBytes;
    if (elect) bulk_wait_group_read<1>();  // the store that last used `buf` has read it
    named_barrier_sync(1, 128);
    uint32_t v[2][32];
    tmem_ld_32x32b_x32(taddr + c, v[0]);
    tmem_ld_32x32b_x32(taddr + c + 32, v[1]);
    tmem_wait_ld();
    epilogue_stage_store<BF16>(tmC, buf, v, rl, elect, col_base + c, row0);
  }
}

template <int BN, bool B_MN, bool SWAP, bool HILO, bool RESID, bool BF16>
__global__ void __launch_bounds__(kThreads, SWAP ? 2 : 1)  // SWAP: two CTAs per SM
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using Cfg = TcCfg<BN, SWAP>;
  constexpr int ST = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* epi_stage = smem + ST * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) TC_TRACE(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) TC_TRACE(1);
  const int64_t num_tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  const int z = static_cast<int>(blockIdx.z);
  const int64_t kb0 = static_cast<int64_t>(z) * p.kb_per_split;
  const int64_t kb1 = (kb0 + p.kb_per_split < p.num_kb) ? kb0 + p.kb_per_split : p.num_kb;
  const bool have_k = kb1 > kb0;
  const int64_t t_begin = blockIdx.x;
  const int64_t t_step = (p.split > 1) ? num_tiles : gridDim.x;  // split: one tile per CTA
  // Set-up done: let the next kernel start launching, then wait for the previous
  // one (no operand or output is read or written before the wait).
  pdl_trigger();
  if constexpr (SWAP) {
    // The weight tiles (operand A here) never depend on the preceding kernel --
    // typically the small activation pre-pass, which leaves most SMs free:
    // pull this CTA's first ST weight tiles into L2 meanwhile.  L2 is coherent,
    // so this cannot return stale data; the TMA loads after the wait hit L2.
    if (warp == 0 && lane == 0 && have_k && t_begin < num_tiles) {
      int tm, tn;
      tile_coords(t_begin, p.tiles_m, p.tiles_n, tm, tn);
      const int64_t kend = (kb1 < kb0 + ST) ? kb1 : kb0 + ST;
      for (int64_t kb = kb0; kb < kend; ++kb)
        tma_prefetch_2d(&tmA, static_cast<int32_t>(kb * kBK), tm * kBM);
    }
  }
  pdl_wait();

  constexpr uint32_t kIdesc = umma_idesc_f16(kBM, BN, BF16, false, B_MN);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && have_k) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = t_begin; ok && t < num_tiles; t += t_step) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
        for (int64_t kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t s = it % ST;
          const uint32_t ph = (it / ST) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, p.limit_ns, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          if (it == 0) TC_TRACE(2);
          tma_load_2d(sa, &tmA, &full[s], static_cast<int32_t>(kb * kBK), tm * kBM);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              tma_load_2d(sb + j * 8192, &tmB, &full[s], tn * BN + j * 64,
                          static_cast<int32_t>(kb * kBK));
            }
          } else {
            tma_load_2d(sb, &tmB, &full[s], static_cast<int32_t>(kb * kBK), tn * BN);
          }
        }
      }
    }
    __syncwarp();  // reconverge warp 0 before the CTA-wide barrier below
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int64_t t = t_begin; ok && t < num_tiles; t += t_step, ++tl) {
        const uint32_t a = tl & 1u;
        const uint32_t aph = (tl >> 1) & 1u;
        if (!mbar_wait(&tempty[a], aph ^ 1u, p.limit_ns, p.err)) break;
        tc_fence_after();
        if (!have_k) {  // empty K range of this cluster rank: the partial is zero
          mbar_arrive(&tfull[a]);
          continue;
        }
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int64_t kb = kb0; kb < kb1; ++kb, ++it) {
          // SWAP: k-block i feeds accumulator i % 4 (first use overwrites).
          const uint32_t i = static_cast<uint32_t>(kb - kb0);
          const uint32_t d_acc = SWAP ? tmem_base + (i & 3u) * BN : d_tmem;
          const bool first = SWAP ? (i < 4u) : (kb == kb0);
          const uint32_t s = it % ST;
          const uint32_t ph = (it / ST) & 1u;
          if (!mbar_wait(&full[s], ph, p.limit_ns, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (it == 0) TC_TRACE(3);
          const uint32_t sa = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = umma_desc_sw128(sa + kk * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (B_MN) {
              bdesc = umma_desc_sw128(sb + kk * 2048, 8192, 1024);
            } else {
              bdesc = umma_desc_sw128(sb + kk * 32, 16, 1024);
            }
            umma_f16(d_acc, adesc, bdesc, kIdesc, (!first || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        TC_TRACE(4);
        umma_commit(&tfull[a]);
      }
    }
    __syncwarp();  // reconverge warp 1 (its lane 0 issued the MMAs)
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int rl = q * 32 + lane;
    uint32_t tl = 0;
    uint32_t epi_chunk = 0;
    for (int64_t t = t_begin; t < num_tiles; t += t_step, ++tl) {
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
      const uint32_t a = tl & 1u;
      const uint32_t aph = (tl >> 1) & 1u;
      if (!mbar_wait(&tfull[a], aph, p.limit_ns, p.err)) break;
      tc_fence_after();
      if (threadIdx.x == 64) TC_TRACE(5);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * BN;
      // 16 accumulator columns [c, c+16) of this thread's row; in SWAP mode the sum
      // of the accumulators that received k-blocks, in fixed order.
      const int nacc = SWAP ? static_cast<int>((kb1 - kb0) < 4 ? (kb1 - kb0) : 4) : 1;
      auto ld16 = [&](int c, float (&f)[16]) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(v[i]);
        if constexpr (SWAP) {
          for (int j = 1; j < nacc; ++j) {
            tmem_ld_32x32b_x16(taddr + j * BN + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) f[i] += __uint_as_float(v[i]);
          }
        }
      };

      if (p.split > 1) {
        // Park the FP32 partial in shared memory (the pipeline ring is idle now).
        // Each chunk's loads from all the accumulators go out before one wait,
        // and are added in accumulator order (as ld16 does).
        float* P = reinterpret_cast<float*>(smem);
        constexpr int CW = 16;  // 4 x 16 registers in flight: two CTAs per SM still fit
        const int na = SWAP ? nacc : 1;
#pragma unroll 1
        for (int c = 0; c < BN; c += CW) {
          uint32_t v[4][CW];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j < na) tmem_ld_32x32b_x16(taddr + j * BN + c, v[j]);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < CW; ++i) {
            float f = __uint_as_float(v[0][i]);
#pragma unroll
            for (int j = 1; j < 4; ++j)
              if (j < na) f += __uint_as_float(v[j][i]);
            P[rl * Cfg::kPartialPitch + c + i] = have_k ? f : 0.0f;
          }
        }
      } else if constexpr (SWAP) {
        if constexpr (HILO) {
          // Columns j and j + half_b hold the two parts of activation row j.
          const int hb = p.half_b;
          float f[BN];
#pragma unroll
          for (int c = 0; c < BN; c += 16) {
            float g16[16];
            ld16(c, g16);
#pragma unroll
            for (int i = 0; i < 16; ++i) f[c + i] = g16[i];
          }
#pragma unroll
          for (int j = 0; j < BN / 2; ++j) {
            if (j < hb) emit<true, RESID, BF16>(p, tm, tn, rl, j, BN, f[j] + f[j + hb]);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            float f[16];
            ld16(c, f);
#pragma unroll
            for (int i = 0; i < 16; ++i) emit<true, RESID, BF16>(p, tm, tn, rl, c + i, BN, f[i]);
          }
        }
      } else if (!RESID && !SWAP && p.tma_epi) {
        if constexpr (!RESID && !SWAP) {
          epilogue_tma_tile<BN, BF16>(&tmC, epi_stage, taddr, rl, warp == 2 && lane == 0,
                                      tn * BN, tm * kBM, epi_chunk);
        }
      } else {
        const int64_t row = static_cast<int64_t>(tm) * kBM + rl;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c, v);
          tmem_wait_ld();
          const int64_t col0 = static_cast<int64_t>(tn) * BN + c;
          if (row < p.out_rows) {
            float f[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
            if (p.vec_out && col0 + 32 <= p.out_cols) {
              const int64_t base = row * p.ldo + col0;
              if constexpr (RESID) {
                const uint4* rp = reinterpret_cast<const uint4*>(
                    reinterpret_cast<const uint16_t*>(p.resid) + base);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                  const uint4 rv = rp[g];
                  const uint16_t* rh = reinterpret_cast<const uint16_t*>(&rv);
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    float r;
                    if constexpr (BF16) {
                      r = __uint_as_float(static_cast<uint32_t>(rh[i]) << 16);
                    } else {
                      r = __half2float(__ushort_as_half(rh[i]));
                    }
                    f[g * 8 + i] += r;
                  }
                }
              }
              uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base);
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                uint4 o;
                o.x = pack2<BF16>(f[g * 8 + 0], f[g * 8 + 1]);
                o.y = pack2<BF16>(f[g * 8 + 2], f[g * 8 + 3]);
                o.z = pack2<BF16>(f[g * 8 + 4], f[g * 8 + 5]);
                o.w = pack2<BF16>(f[g * 8 + 6], f[g * 8 + 7]);
                op[g] = o;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) emit<false, RESID, BF16>(p, tm, tn, rl, c + i, BN, f[i]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[a]);
    }
    if (warp == 2 && lane == 0) bulk_wait_group<0>();  // TMA stores complete before exit
  }

  __syncthreads();
  if (threadIdx.x == 0) TC_TRACE(6);

  if (p.split > 1) {
    // Sum the S partials of this tile in rank order; CTA z finishes rows z, z+S, ...
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    int tm, tn;
    tile_coords(t_begin, p.tiles_m, p.tiles_n, tm, tn);
    const float* P = reinterpret_cast<const float*>(smem);
    const int S = p.split;
    const int my_rows = (kBM - z + S - 1) / S;
    const int cols = HILO ? p.half_b : BN;
    if (cols % 4 == 0 && (!HILO || p.half_b % 4 == 0)) {
      // Four adjacent columns per thread: one 16-byte DSMEM load per rank (two
      // with HILO), all ranks' loads issued before the sums, which keep the
      // rank order (hi then lo per rank) of the scalar form below.
      const int c4 = cols / 4;
      for (int e = threadIdx.x; e < my_rows * c4; e += kThreads) {
        const int r = z + S * (e / c4);
        const int j = (e % c4) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q0 = 0; q0 < 8; q0 += 4) {  // four ranks' loads in flight at a time
          float4 a[4], b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (q0 + i < S) {
              const float* peer = cluster.map_shared_rank(P, q0 + i) + r * Cfg::kPartialPitch + j;
              a[i] = *reinterpret_cast<const float4*>(peer);
              if constexpr (HILO) b[i] = *reinterpret_cast<const float4*>(peer + p.half_b);
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (q0 + i < S) {
              v.x += a[i].x; v.y += a[i].y; v.z += a[i].z; v.w += a[i].w;
              if constexpr (HILO) { v.x += b[i].x; v.y += b[i].y; v.z += b[i].z; v.w += b[i].w; }
            }
          }
        }
        emit<SWAP, RESID, BF16>(p, tm, tn, r, j, BN, v.x);
        emit<SWAP, RESID, BF16>(p, tm, tn, r, j + 1, BN, v.y);
        emit<SWAP, RESID, BF16>(p, tm, tn, r, j + 2, BN, v.z);
        emit<SWAP, RESID, BF16>(p, tm, tn, r, j + 3, BN, v.w);
      }
    } else {
      for (int e = threadIdx.x; e < my_rows * cols; e += kThreads) {
        const int r = z + S * (e / cols);
        const int j = e % cols;
        float v = 0.0f;
        for (int qr = 0; qr < S; ++qr) {
          const float* peer = cluster.map_shared_rank(P, qr);
          v += peer[r * Cfg::kPartialPitch + j];
          if constexpr (HILO) v += peer[r * Cfg::kPartialPitch + j + p.half_b];
        }
        emit<SWAP, RESID, BF16>(p, tm, tn, r, j, BN, v);
      }
    }
    cluster.sync();
  }

  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
#ifdef ENGINE_TC_TRACE
  if (threadIdx.x == 0 && p.trace) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    TC_TRACE(7);
    p.trace[(blockIdx.x + gridDim.x * blockIdx.z) * 8 + 7] =
        (p.trace[(blockIdx.x + gridDim.x * blockIdx.z) * 8 + 7] << 8) | smid;
  }
#endif
}

// ------------------------------------------------------------ 2-SM (M = 256) GEMM
//
// A CTA pair (cluster of 2) computes a 256 x BN output tile with
// tcgen05.mma.cta_group::2: CTA r holds rows [128r, 128r+128) of the A tile and
// columns [r*BN/2, (r+1)*BN/2) of the B tile in its own shared memory, and rows
// [128r, 128r+128) of the FP32 accumulator in its own TMEM.  Per SM this halves
// the shared-memory operand bandwidth (and the L2 operand traffic) of a
// 128 x BN tile.  Roles as in gemm_tc_kernel, with these cross-CTA links:
//   * both producers wait on their own `empty` barrier, then load their halves;
//     the leader (rank 0) arms its `full` barrier for BOTH CTAs' bytes and the
//     peer's TMA completes on the leader's barrier (shared::cluster address);
//   * the leader's MMA thread issues the 2-SM MMA and commits each stage (and
//     each finished accumulator) to the barriers of BOTH CTAs -- two plain
//     commits, one per CTA;
//   * both epilogues drain their own TMEM lanes and arrive on the leader's
//     `tempty` barrier (count 8 = 4 warps x 2 CTAs).
// No TMA multicast is used.

template <int BN>
struct Tc2Cfg {
  static constexpr int kABytes = 128 * kBK * 2;       // this CTA's 128 rows of A
  static constexpr int kBBytes = (BN / 2) * kBK * 2;  // this CTA's BN/2 rows / columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = ENGINE_TC2_STAGES > 0 ? ENGINE_TC2_STAGES : ((BN >= 256) ? 6 : 8);
  static constexpr int kTmemCols = pow2_at_least(2 * BN);
  static constexpr int kEpiBytes = 2 * kEpiStageBytes;  // TMA-store staging
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int BN, bool B_MN, bool RESID, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using Cfg = Tc2Cfg<BN>;
  constexpr int ST = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* epi_stage = smem + ST * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint32_t* sk_flag = tmem_slot + 1;  // stream-K: this CTA stores the tile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const bool leader = rank == 0;
  if (threadIdx.x == 0) TC_TRACE(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);   // leader: its producer's expect_tx arrival
      mbar_init(&empty[s], 1);  // one commit from the leader's MMA thread
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // leader: 4 epilogue warps x 2 CTAs
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_2sm(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) TC_TRACE(1);

  const int64_t pair = blockIdx.x >> 1;
  const int64_t npairs = gridDim.x >> 1;
  const int64_t nkb = p.num_kb;
  constexpr uint32_t kIdesc = umma_idesc_f16(256, BN, BF16, false, B_MN);

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      uint32_t it = 0;
      bool ok = true;
      TcSched sch(p, pair, npairs);
      TcWork w;
      while (ok && sch.next(p, npairs, w)) {
        int tm, tn;
        tile_coords(w.tile, p.tiles_m, p.tiles_n, tm, tn);
        for (int64_t kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % ST;
          const uint32_t ph = (it / ST) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, p.limit_ns, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
          const uint32_t fbar = full_leader0 + s * 8;
          tma_load_2d_2sm(sa, &tmA, fbar, static_cast<int32_t>(kb * kBK),
                          tm * 256 + static_cast<int>(rank) * 128);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) {
              tma_load_2d_2sm(sb + j * 8192, &tmB, fbar,
                              tn * BN + static_cast<int>(rank) * (BN / 2) + j * 64,
                              static_cast<int32_t>(kb * kBK));
            }
          } else {
            tma_load_2d_2sm(sb, &tmB, fbar, static_cast<int32_t>(kb * kBK),
                            tn * BN + static_cast<int>(rank) * (BN / 2));
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t empty_peer0 = mapa_shared(smem_u32(&empty[0]), 1);
      const uint32_t empty_self0 = mapa_shared(smem_u32(&empty[0]), 0);
      const uint32_t tfull_peer0 = mapa_shared(smem_u32(&tfull[0]), 1);
      const uint32_t tfull_self0 = mapa_shared(smem_u32(&tfull[0]), 0);
      uint32_t it = 0, tl = 0;
      bool ok = true;
      TcSched sch(p, pair, npairs);
      TcWork w;
      for (; ok && sch.next(p, npairs, w); ++tl) {
        const uint32_t a = tl & 1u;
        const uint32_t aph = (tl >> 1) & 1u;
        if (!mbar_wait(&tempty[a], aph ^ 1u, p.limit_ns, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
#ifdef ENGINE_TC_TRACE
        if (w.tile >= p.dp_tiles && p.trace && p.trace[blockIdx.x * 8 + 2] == 0) TC_TRACE(2);
#endif
        for (int64_t kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const uint32_t s = it % ST;
          const uint32_t ph = (it / ST) & 1u;
          if (!mbar_wait(&full[s], ph, p.limit_ns, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = umma_desc_sw128(sa + kk * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (B_MN) {
              bdesc = umma_desc_sw128(sb + kk * 2048, 8192, 1024);
            } else {
              bdesc = umma_desc_sw128(sb + kk * 32, 16, 1024);
            }
            umma_f16_2sm(d_tmem, adesc, bdesc, kIdesc, (kb > w.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_2sm(empty_self0 + s * 8);
          umma_commit_2sm(empty_peer0 + s * 8);
        }
        if (!ok) break;
        umma_commit_2sm(tfull_self0 + a * 8);
        umma_commit_2sm(tfull_peer0 + a * 8);
      }
      TC_TRACE(3);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int rl = q * 32 + lane;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    uint32_t tl = 0;
    uint32_t epi_chunk = 0;
    TcSched sch(p, pair, npairs);
    TcWork w;
    for (; sch.next(p, npairs, w); ++tl) {
      int tm, tn;
      tile_coords(w.tile, p.tiles_m, p.tiles_n, tm, tn);
      const uint32_t a = tl & 1u;
      const uint32_t aph = (tl >> 1) & 1u;
      if (!mbar_wait(&tfull[a], aph, p.limit_ns, p.err)) break;
      tc_fence_after();
      if (warp == 2 && lane == 0) TC_TRACE(5);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * BN;
      const int64_t row = static_cast<int64_t>(tm) * 256 + static_cast<int64_t>(rank) * 128 + rl;
      const float* other = nullptr;  // stream-K: the other pair's partial of this tile
      if (w.sk_tile >= 0) {
        // The second of the tile's two pairs to arrive stores the tile.  If the
        // other pair has already parked its partial, this CTA stores the tile
        // at once; otherwise it parks its own partial and arrives, and whichever
        // arrival comes second does the store.
        unsigned long long* cnt = p.ws_cnt + w.sk_tile * 2 + rank;
        if (warp == 2 && lane == 0) {
          unsigned long long v;
          asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(cnt) : "memory");
          const bool second = static_cast<uint32_t>(v) == 1u;
          if (second) sk_reset(cnt);
          *sk_flag = second ? 1u : 0u;
        }
        named_barrier_sync(1, 128);
        if (*reinterpret_cast<volatile uint32_t*>(sk_flag) == 0u) {
          float* mine = sk_slot<BN>(p, pair, sk_slot_of(p, pair, w.sk_tile, npairs), rank);
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(taddr + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __stcg(sk_quad(mine, (c >> 2) + j, rl),
                     make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
            }
          }
          named_barrier_sync(1, 128);
          if (warp == 2 && lane == 0) {
            const uint32_t n = sk_arrive(cnt);
            if (n == 2) sk_reset(cnt);
            *sk_flag = (n == 2) ? 1u : 0u;
          }
          named_barrier_sync(1, 128);
          if (*reinterpret_cast<volatile uint32_t*>(sk_flag) == 0u) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader0 + a * 8);
            continue;
          }
        }
        if (warp == 2 && lane == 0) TC_TRACE(6);
        const int64_t first = sk_owner(p, w.sk_tile * nkb, npairs);
        const int64_t q_other = (first == pair) ? pair + 1 : first;
        other = sk_slot<BN>(p, q_other, sk_slot_of(p, q_other, w.sk_tile, npairs), rank);
      }
      if constexpr (!RESID) {
        if (p.tma_epi) {
          epilogue_tma_tile<BN, BF16>(&tmC, epi_stage, taddr, rl, warp == 2 && lane == 0,
                                      tn * BN, tm * 256 + static_cast<int>(rank) * 128,
                                      epi_chunk, other);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader0 + a * 8);
          continue;
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        float4 x[8];
        if (other != nullptr) sk_load32(x, other, c, rl);
        tmem_ld_32x32b_x32(taddr + c, v);
        tmem_wait_ld();
        if (other != nullptr) sk_add32(v, x);
        const int64_t col0 = static_cast<int64_t>(tn) * BN + c;
        if (row < p.out_rows) {
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
          if (p.vec_out && col0 + 32 <= p.out_cols) {
            const int64_t base = row * p.ldo + col0;
            if constexpr (RESID) {
              const uint4* rp = reinterpret_cast<const uint4*>(
                  reinterpret_cast<const uint16_t*>(p.resid) + base);
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                const uint4 rv = rp[g];
                const uint16_t* rh = reinterpret_cast<const uint16_t*>(&rv);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  float r;
                  if constexpr (BF16) {
                    r = __uint_as_float(static_cast<uint32_t>(rh[i]) << 16);
                  } else {
                    r = __half2float(__ushort_as_half(rh[i]));
                  }
                  f[g * 8 + i] += r;
                }
              }
            }
            uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 o;
              o.x = pack2<BF16>(f[g * 8 + 0], f[g * 8 + 1]);
              o.y = pack2<BF16>(f[g * 8 + 2], f[g * 8 + 3]);
              o.z = pack2<BF16>(f[g * 8 + 4], f[g * 8 + 5]);
              o.w = pack2<BF16>(f[g * 8 + 6], f[g * 8 + 7]);
              op[g] = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int64_t cc = col0 + i;
              if (cc < p.out_cols) {
                float vv = f[i];
                if constexpr (RESID) vv += load16<BF16>(p.resid, row * p.ldo + cc);
                store16<BF16>(p.out, row * p.ldo + cc, vv);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + a * 8);
    }
    if (warp == 2 && lane == 0) {
      bulk_wait_group<0>();  // TMA stores complete before exit
      TC_TRACE(4);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, Cfg::kTmemCols);
  }
#ifdef ENGINE_TC_TRACE
  if (threadIdx.x == 0 && p.trace) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    TC_TRACE(7);
    p.trace[blockIdx.x * 8 + 7] = (p.trace[blockIdx.x * 8 + 7] << 8) | smid;
  }
#endif
}

// ------------------------------------------------------------------ host side

template <int BN, bool B_MN, bool SWAP, bool HILO, bool RESID, bool BF16>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
              const TcParams& p, int grid_x, cudaStream_t stream) {
  using Cfg = TcCfg<BN, SWAP>;
  auto kern = gemm_tc_kernel<BN, B_MN, SWAP, HILO, RESID, BF16>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load() & bit) == 0) {
    B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::kSmemBytes));
    configured.fetch_or(bit);
  }
  TcParams q = p;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(grid_x), 1, static_cast<unsigned>(q.split));
  attr[0].val.clusterDim.z = static_cast<unsigned>(q.split);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  B200_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, q));
  return ENGINE_OK;
}

template <int BN, bool B_MN, bool RESID, bool BF16>
int launch_tc2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
               const TcParams& p, int grid_x, cudaStream_t stream) {
  using Cfg = Tc2Cfg<BN>;
  auto kern = gemm_tc2_kernel<BN, B_MN, RESID, BF16>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load() & bit) == 0) {
    B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::kSmemBytes));
    configured.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid_x), 1, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  B200_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, p));
  return ENGINE_OK;
}

template <int BN, bool B_MN, bool SWAP, bool HILO, bool BF16>
int launch_tc_r(bool resid, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                const TcParams& p, int grid_x, cudaStream_t stream) {
  return resid ? launch_tc<BN, B_MN, SWAP, HILO, true, BF16>(ta, tb, tc, p, grid_x, stream)
               : launch_tc<BN, B_MN, SWAP, HILO, false, BF16>(ta, tb, tc, p, grid_x, stream);
}

int env_int(const char* name, int dflt) {
  const char* e = std::getenv(name);
  if (e == nullptr || e[0] == '\0') return dflt;
  return static_cast<int>(std::strtol(e, nullptr, 10));
}

// Stream-K workspace of the 2-SM kernel, one per (device, stream): calls on one
// stream run one after another (every access follows the kernel's
// griddepcontrol.wait), so their partial slots and counters never overlap;
// calls on different streams get different workspaces.  Sized for the largest
// grid (two slots per CTA pair, BN = 256) and kept for the life of the
// process.  Counters start at zero and every completed launch leaves them at
// zero, so a CUDA graph may replay a captured launch.  The first call on a
// stream allocates; a call made during stream capture before that falls back
// to whole-tile scheduling.
struct SkWorkspace {
  float* parts = nullptr;
  unsigned long long* cnt = nullptr;
  size_t cnt_bytes = 0;
};

std::mutex g_sk_mu;
std::map<std::pair<int, cudaStream_t>, SkWorkspace> g_sk_spaces;

bool sk_workspace(int dev, cudaStream_t stream, int max_pairs, float** parts,
                  unsigned long long** cnt) {
  std::lock_guard<std::mutex> lk(g_sk_mu);
  auto& spaces = g_sk_spaces;
  SkWorkspace& w = spaces[std::make_pair(dev, stream)];
  if (w.parts == nullptr) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      return false;
    // Partial slots: 2 per pair x 2 CTAs x 128 x 256 FP32.  Counters: one per
    // (stream-K tile, CTA rank); the stream-K region has fewer than 2 x pairs tiles.
    const size_t part_bytes = static_cast<size_t>(max_pairs) * 2 * 2 * 128 * 256 * sizeof(float);
    const size_t cnt_bytes = static_cast<size_t>(2 * max_pairs) * 2 * sizeof(unsigned long long);
    void* mem = nullptr;
    if (cudaMalloc(&mem, part_bytes + cnt_bytes) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (cudaMemset(reinterpret_cast<uint8_t*>(mem) + part_bytes, 0, cnt_bytes) != cudaSuccess) {
      cudaFree(mem);
      cudaGetLastError();
      return false;
    }
    w.parts = reinterpret_cast<float*>(mem);
    w.cnt = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(mem) + part_bytes);
    w.cnt_bytes = cnt_bytes;
  }
  *parts = w.parts;
  *cnt = w.cnt;
  return true;
}

// 16-bit GEMM on CUDA cores for shapes TMA cannot describe (row pitch not a
// multiple of 16 bytes, misaligned base).  FP32 accumulate; same epilogue rules.
template <bool BF16>
__global__ void __launch_bounds__(256) gemm16_simt_kernel(const void* __restrict__ A,
                                                          const void* __restrict__ B,
                                                          const void* __restrict__ R,
                                                          void* __restrict__ C, int64_t M,
                                                          int64_t N, int64_t K, int b_kmajor) {
  __shared__ float As[16][17];
  __shared__ float Bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row = static_cast<int64_t>(blockIdx.y) * 16 + ty;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * 16 + tx;
  float acc = 0.0f;
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    const int64_t ka = k0 + tx;
    As[ty][tx] = (row < M && ka < K) ? load16<BF16>(A, row * K + ka) : 0.0f;
    const int64_t kb = k0 + ty;
    float bv = 0.0f;
    if (kb < K && col < N) bv = b_kmajor ? load16<BF16>(B, col * K + kb) : load16<BF16>(B, kb * N + col);
    Bs[ty][tx] = bv;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc = fmaf(As[ty][i], Bs[i][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) {
    float v = acc;
    if (R != nullptr) v += load16<BF16>(R, row * N + col);
    store16<BF16>(C, row * N + col, v);
  }
}

}  // namespace

int gemm_tc_general(const void* A, const void* B, const void* residual, void* C, int64_t M,
                    int64_t N, int64_t K, bool bf16, bool b_kmajor, bool hilo, int half_b,
                    cudaStream_t stream);

int gemm_tc(const void* A, const void* B, const void* residual, void* C, int64_t M, int64_t N,
            int64_t K, bool bf16, bool b_kmajor, cudaStream_t stream) {
  return gemm_tc_general(A, B, residual, C, M, N, K, bf16, b_kmajor, false, 0, stream);
}

int gemm_tc_dispatch(const void* A, const void* B, const void* residual, void* C, int64_t M,
                     int64_t N, int64_t K, bool bf16, bool b_kmajor, bool hilo, int half_b,
                     cudaStream_t stream);

void sk_workspace_reset(int dev) {
  std::lock_guard<std::mutex> lk(g_sk_mu);
  for (auto& kv : g_sk_spaces) {
    if (kv.first.first == dev && kv.second.cnt != nullptr)
      cudaMemset(kv.second.cnt, 0, kv.second.cnt_bytes);
  }
}

int gemm_tc_general(const void* A, const void* B, const void* residual, void* C, int64_t M,
                    int64_t N, int64_t K, bool bf16, bool b_kmajor, bool hilo, int half_b,
                    cudaStream_t stream) {
  const int rc = gemm_tc_dispatch(A, B, residual, C, M, N, K, bf16, b_kmajor, hilo, half_b, stream);
  if (rc != ENGINE_OK) return rc;
  return check_launch("matmul/linear (tcgen05)");
}


/// With hilo=true, A holds 2*half_b activation rows (FP16 roundings, then the
/// FP16 roundings of the remainders) of a batch padded to half_b rows, b_kmajor
/// must be true, and the result rows are the first `M` rows of C.
int gemm_tc_dispatch(const void* A, const void* B, const void* residual, void* C, int64_t M,
                    int64_t N, int64_t K, bool bf16, bool b_kmajor, bool hilo, int half_b,
                    cudaStream_t stream) {
  // TMA tile coordinates and tile counts are 32-bit.
  B200_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
               "matmul: dimension too large (each must be below 2^31)");
  const CUtensorMapDataType dt =
      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uintptr_t pa = reinterpret_cast<uintptr_t>(A), pb = reinterpret_cast<uintptr_t>(B);
  const bool tma_ok = (K % 8 == 0) && (pa % 16 == 0) && (pb % 16 == 0) &&
                      (b_kmajor || (N % 8 == 0));
  if (!tma_ok) {
    B200_REQUIRE(!hilo, "internal: hi/lo activations need 16-byte aligned rows");
    dim3 grid(static_cast<unsigned>((N + 15) / 16), static_cast<unsigned>((M + 15) / 16));
    B200_REQUIRE(grid.y <= 65535, "matmul: M too large for the fallback kernel");
    if (bf16) {
      gemm16_simt_kernel<true><<<grid, 256, 0, stream>>>(A, B, residual, C, M, N, K, b_kmajor);
    } else {
      gemm16_simt_kernel<false><<<grid, 256, 0, stream>>>(A, B, residual, C, M, N, K, b_kmajor);
    }
    return ENGINE_OK;
  }

  const int sms = sm_count();
  TcParams p = {};
  p.K = K;
  p.num_kb = (K + kBK - 1) / kBK;
  p.out = C;
  p.resid = residual;
  p.ldo = N;
  p.out_rows = M;
  p.out_cols = N;
  p.err = device_error_word();
  p.limit_ns = wait_limit_ns();
#ifdef ENGINE_TC_TRACE
  {
    const char* e = std::getenv("ENGINE_TC_TRACE_PTR");
    p.trace = e ? reinterpret_cast<unsigned long long*>(std::strtoull(e, nullptr, 0)) : nullptr;
  }
#endif
  p.vec_out = (N % 8 == 0) && (reinterpret_cast<uintptr_t>(C) % 16 == 0) &&
              (residual == nullptr || reinterpret_cast<uintptr_t>(residual) % 16 == 0);
  const bool resid = residual != nullptr;
  // Output tensor map for the TMA-store epilogue (general GEMM paths only).
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  p.tma_epi = 0;
  static const int tma_epi_env = env_int("ENGINE_TC_TMA_EPI", 1);
  auto enable_tma_out = [&]() {
    if (tma_epi_env != 0 && !resid && (N % 8 == 0) && (reinterpret_cast<uintptr_t>(C) % 16 == 0) &&
        make_tmap_2d(&tc, C, dt, 2, static_cast<uint64_t>(M), static_cast<uint64_t>(N),
                     static_cast<uint64_t>(N), 128, 64)) {
      p.tma_epi = 1;
    }
  };

  // Small batch against [N,K] weights: weights are the 128-row UMMA operand.
  const int64_t act_rows = hilo ? 2 * static_cast<int64_t>(half_b) : M;
  static const int swap_max = env_int("ENGINE_TC_SWAP_MAX_M", 64);
  if (b_kmajor && act_rows <= 64 && (hilo || M <= swap_max)) {
    int bn = 16;
    while (bn < act_rows) bn <<= 1;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, B, dt, 2, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                      static_cast<uint64_t>(K), kBM, kBK))
      return ENGINE_ERR_UNSUPPORTED;
    if (!make_tmap_2d(&tb, A, dt, 2, static_cast<uint64_t>(act_rows), static_cast<uint64_t>(K),
                      static_cast<uint64_t>(K), static_cast<uint32_t>(bn), kBK))
      return ENGINE_ERR_UNSUPPORTED;
    p.tiles_m = static_cast<int>((N + kBM - 1) / kBM);
    p.tiles_n = 1;
    p.half_b = half_b;
    const int tiles = p.tiles_m;
    // Split-K over a cluster of S CTAs when the weight tiles alone cannot cover
    // the SMs (two CTAs fit per SM in this mode): the largest S <= 8 with at
    // least four k-blocks per split and tiles x S within 85% of the 2-per-SM
    // slots.  A B200 sweep (M = 16; N x K = 6144x4096, 4096x4096, 28672x4096,
    // 4096x14336) found that point fastest on every shape.  Clusters that do
    // not all fit at once only wait for a slot: no cluster depends on another.
    int S = 1;
    if (tiles > 0) {
      S = static_cast<int>((static_cast<int64_t>(sms) * 2 * 85 / 100) / tiles);
      if (S > 8) S = 8;
      const int64_t kmax = p.num_kb / 4;
      if (S > kmax) S = static_cast<int>(kmax);
      if (S < 1) S = 1;
    }
    static const int split_env = env_int("ENGINE_TC_SPLIT", 0);
    if (split_env > 0) S = split_env > 8 ? 8 : split_env;
    p.split = S;
    p.kb_per_split = (p.num_kb + S - 1) / S;
    const int grid = tiles;
    if (hilo) {
      switch (bn) {
        case 16: return bf16 ? launch_tc_r<16, false, true, true, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<16, false, true, true, false>(resid, ta, tb, tc, p, grid, stream);
        case 32: return bf16 ? launch_tc_r<32, false, true, true, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<32, false, true, true, false>(resid, ta, tb, tc, p, grid, stream);
        default: return bf16 ? launch_tc_r<64, false, true, true, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<64, false, true, true, false>(resid, ta, tb, tc, p, grid, stream);
      }
    }
    switch (bn) {
      case 16: return bf16 ? launch_tc_r<16, false, true, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<16, false, true, false, false>(resid, ta, tb, tc, p, grid, stream);
      case 32: return bf16 ? launch_tc_r<32, false, true, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<32, false, true, false, false>(resid, ta, tb, tc, p, grid, stream);
      default: return bf16 ? launch_tc_r<64, false, true, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<64, false, true, false, false>(resid, ta, tb, tc, p, grid, stream);
    }
  }
  B200_REQUIRE(!hilo, "internal: hi/lo activations are limited to 32 rows");

  // Large GEMMs: 2-SM tcgen05 (256 x BN tiles over CTA pairs).
  static const int two_sm_env = env_int("ENGINE_TC_2SM", 1);
  if (two_sm_env != 0 && M >= 256 && N >= 256) {
    static const int bn2_env = env_int("ENGINE_TC2_BN", 0);
    const int bn2 = (bn2_env == 128) ? 128 : 256;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, dt, 2, static_cast<uint64_t>(M), static_cast<uint64_t>(K),
                      static_cast<uint64_t>(K), 128, kBK))
      return ENGINE_ERR_UNSUPPORTED;
    if (b_kmajor) {
      if (!make_tmap_2d(&tb, B, dt, 2, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                        static_cast<uint64_t>(K), static_cast<uint32_t>(bn2 / 2), kBK))
        return ENGINE_ERR_UNSUPPORTED;
    } else {
      if (!make_tmap_2d(&tb, B, dt, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                        static_cast<uint64_t>(N), kBK, 64))
        return ENGINE_ERR_UNSUPPORTED;
    }
    enable_tma_out();
    p.tiles_m = static_cast<int>((M + 255) / 256);
    p.tiles_n = static_cast<int>((N + bn2 - 1) / bn2);
    p.split = 1;
    p.kb_per_split = p.num_kb;
    p.half_b = 0;
    const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
    const int pairs = static_cast<int>(tiles < sms / 2 ? tiles : sms / 2);
    const int grid = 2 * pairs;
    // Whole tiles round-robin, unless the last wave would leave between 1/16 and
    // 1/2 of the pairs idle: then all but one full wave stays round-robin and
    // the rest (between `pairs` and 2 * `pairs` tiles) is split along K evenly.
    // A last wave at least half full runs faster as whole tiles (B200, CUDA
    // graph: X[512,4096] W[14336,4096]^T, 112 tiles on 74 pairs, 54.7 against
    // 60.3 us split), while a nearly empty one gains from the split (S = 1024:
    // 97.6 against 101 us; S = 2048: 173 against 181 us).
    p.dp_tiles = tiles;
    p.sk_iters = 0;
    static const int streamk_env = env_int("ENGINE_TC_STREAMK", 1);
    const int64_t waves = tiles / pairs;
    const int64_t rem = tiles % pairs;
    if (streamk_env != 0 && waves >= 1 && rem != 0 && (pairs - rem) * 16 >= pairs &&
        2 * rem < pairs && p.num_kb >= 8) {
      int dev = 0;
      B200_CUDA(cudaGetDevice(&dev));
      if (sk_workspace(dev, stream, sms / 2, &p.ws, &p.ws_cnt)) {
        p.dp_tiles = (waves - 1) * pairs;
        p.sk_iters = (tiles - p.dp_tiles) * p.num_kb;
      }
    }
    if (bn2 == 128) {
      if (b_kmajor) return bf16 ? (resid ? launch_tc2<128, false, true, true>(ta, tb, tc, p, grid, stream) : launch_tc2<128, false, false, true>(ta, tb, tc, p, grid, stream))
                                : (resid ? launch_tc2<128, false, true, false>(ta, tb, tc, p, grid, stream) : launch_tc2<128, false, false, false>(ta, tb, tc, p, grid, stream));
      return bf16 ? (resid ? launch_tc2<128, true, true, true>(ta, tb, tc, p, grid, stream) : launch_tc2<128, true, false, true>(ta, tb, tc, p, grid, stream))
                  : (resid ? launch_tc2<128, true, true, false>(ta, tb, tc, p, grid, stream) : launch_tc2<128, true, false, false>(ta, tb, tc, p, grid, stream));
    }
    if (b_kmajor) return bf16 ? (resid ? launch_tc2<256, false, true, true>(ta, tb, tc, p, grid, stream) : launch_tc2<256, false, false, true>(ta, tb, tc, p, grid, stream))
                              : (resid ? launch_tc2<256, false, true, false>(ta, tb, tc, p, grid, stream) : launch_tc2<256, false, false, false>(ta, tb, tc, p, grid, stream));
    return bf16 ? (resid ? launch_tc2<256, true, true, true>(ta, tb, tc, p, grid, stream) : launch_tc2<256, true, false, true>(ta, tb, tc, p, grid, stream))
                : (resid ? launch_tc2<256, true, true, false>(ta, tb, tc, p, grid, stream) : launch_tc2<256, true, false, false>(ta, tb, tc, p, grid, stream));
  }

  // General persistent GEMM: 128 x BN output tiles.
  static const int bn_env = env_int("ENGINE_TC_BN", 0);
  int bn = bn_env > 0 ? bn_env : (N >= 256 ? 256 : (N > 64 ? 128 : 64));
  if (bn != 64 && bn != 128 && bn != 256) bn = 256;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, dt, 2, static_cast<uint64_t>(M), static_cast<uint64_t>(K),
                    static_cast<uint64_t>(K), kBM, kBK))
    return ENGINE_ERR_UNSUPPORTED;
  if (b_kmajor) {
    if (!make_tmap_2d(&tb, B, dt, 2, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                      static_cast<uint64_t>(K), static_cast<uint32_t>(bn), kBK))
      return ENGINE_ERR_UNSUPPORTED;
  } else {
    // B[K,N]: 64-wide (128-byte) column boxes, 64 k-rows each.
    if (!make_tmap_2d(&tb, B, dt, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                      static_cast<uint64_t>(N), kBK, 64))
      return ENGINE_ERR_UNSUPPORTED;
  }
  enable_tma_out();
  p.tiles_m = static_cast<int>((M + kBM - 1) / kBM);
  p.tiles_n = static_cast<int>((N + bn - 1) / bn);
  p.split = 1;
  p.kb_per_split = p.num_kb;
  p.half_b = 0;
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (b_kmajor) {
    switch (bn) {
      case 64: return bf16 ? launch_tc_r<64, false, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<64, false, false, false, false>(resid, ta, tb, tc, p, grid, stream);
      case 128: return bf16 ? launch_tc_r<128, false, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<128, false, false, false, false>(resid, ta, tb, tc, p, grid, stream);
      default: return bf16 ? launch_tc_r<256, false, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<256, false, false, false, false>(resid, ta, tb, tc, p, grid, stream);
    }
  }
  switch (bn) {
    case 64: return bf16 ? launch_tc_r<64, true, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<64, true, false, false, false>(resid, ta, tb, tc, p, grid, stream);
    case 128: return bf16 ? launch_tc_r<128, true, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<128, true, false, false, false>(resid, ta, tb, tc, p, grid, stream);
    default: return bf16 ? launch_tc_r<256, true, false, false, true>(resid, ta, tb, tc, p, grid, stream) : launch_tc_r<256, true, false, false, false>(resid, ta, tb, tc, p, grid, stream);
  }
}

}  // namespace b200
