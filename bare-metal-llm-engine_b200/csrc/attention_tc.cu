// attention_tc.cu -- attention prefill on the 5th-generation tensor cores
// (tcgen05), FlashAttention-2 style: one pass over the keys with an online
// softmax, S = Q K^T and O += P V on tcgen05 with TMEM accumulators, K / V
// tiles streamed by TMA.
//
// Layouts and arithmetic target are the engine's attention_prefill contract
// (include/engine/kernels.hpp:153, kernels/attention_prefill.cu:329-360): q /
// out [s_q][n_heads][d], k / v [n_kv_heads][kv_head_stride] with key j of a KV
// head at j * d, query head h reading KV head h / (n_heads / n_kv_heads); query
// row i sees keys j <= q_pos_offset + i when causal.  lse[i][h] is the natural
// log-sum-exp of the row's scaled scores.
//
// One CTA owns 128 query rows of one head (grid: q-blocks x heads, the
// q-blocks with the most keys first) and runs 64 + 128 * NS threads in three
// roles.  By default two CTAs share an SM (NB = 1 below: 96 KB of shared
// memory and 256 TMEM columns each); each CTA's chain S -> softmax -> PV is
// serial, and the two chains interleave on the tensor cores.  NB = 3 (one CTA
// per SM, three S / P buffers, two-stage K / V rings) overlaps them inside one
// CTA instead; on B200 it was 17% slower at S = 2048.
//   warp 0      one elected thread issues TMA loads: the Q tile once (3-D map
//               over [s_q][n_heads][d]), then K and V tiles of 128 keys into
//               rings of ST stages (3-D maps over [n_kv_heads][keys][d]; zero
//               fill past s_kv);
//   warp 1      allocates TMEM (NB 128-column S / P buffers and a D-column O
//               accumulator) and one thread issues tcgen05.mma: S[j] = Q K[j]^T
//               into buffer j % NB (A = Q, B = K, both K-major, M = N = 128), and
//               O += P[j] V[j] with A = P[j] read from tensor memory and B = V
//               (MN-major, N = d); S[j] waits for the PV product that last read
//               its buffer (tile j - NB);
//   warps 2..   the softmax, NS threads per query row: warp w reads TMEM lanes
//               32*(w%4)..+31 (its rows) and column group (w-2)/4 of them, so
//               NS warps share each lane quarter (the MUFU and FMA work of a
//               tile spreads over 4*NS warps).  A thread reads its slice of S
//               with tcgen05.ld, masks keys past s_kv and above the causal
//               diagonal; the row max (of the raw scores: the scale c > 0 is
//               folded into one FMA before ex2) is combined across the row's
//               threads through shared memory (bounded mbarrier exchange); it
//               keeps the running max m (base-2 domain) and its partial sum l
//               in FP32 and writes P = exp2(S*c - m) as FP16 pairs with
//               tcgen05.st over the first 64 columns of the same buffer -- no
//               shared-memory round trip and no wait for the previous PV
//               product.  When the row max grew by more than 2^8 it rescales
//               its slice of O in TMEM (tcgen05.ld / st, after PV[j-1]); below
//               that, P <= 2^8 is kept against the old max.  At the end the
//               partial sums are added in column-group order, O is read,
//               divided by l, rounded once to FP16 and stored, and
//               lse = m ln 2 + ln l.
// Tiles of keys entirely above the causal diagonal are never loaded.  The sum l
// is formed from the FP32 probabilities; P enters the tensor cores rounded to
// FP16 (relative error <= 2^-11 per probability).
//
// Every mbarrier wait is bounded (ENGINE_WAIT_TIMEOUT_MS): on expiry the thread
// sets the device error word, abandons its loop and reaches the common teardown.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"

namespace b200 {
namespace {

constexpr int kAtBM = 128;       // query rows per CTA
constexpr int kAtBN = 128;       // keys per tile
// Threads: a producer warp, an MMA warp and 4 * NS softmax warps (NS threads per
// query row).
constexpr int at_threads(int ns) { return 64 + 128 * ns; }
constexpr float kAtRescale = 8.0f;
#ifndef ENGINE_ATTN_NS128
#define ENGINE_ATTN_NS128 2
#endif
#ifndef ENGINE_ATTN_NS64
#define ENGINE_ATTN_NS64 2
#endif
constexpr int kAtSplit128 = ENGINE_ATTN_NS128;  // softmax threads per row, d = 128
constexpr int kAtSplit64 = ENGINE_ATTN_NS64;    // d = 64
#ifndef ENGINE_ATTN_BUFS
#define ENGINE_ATTN_BUFS 1
#endif
constexpr int kAtBufs = ENGINE_ATTN_BUFS;       // S / P buffers (3: one CTA per SM, 1: two)

// NB S / P buffers in TMEM: 3 with one CTA per SM (two-stage K / V rings); 1
// with two CTAs per SM (single K / V stages, 96 KB of shared memory and 256
// TMEM columns each), whose serial S -> softmax -> PV chains interleave.
template <int D, int NB>
struct AtCfg {
  static constexpr int kDH = D / 64;                     // 64-wide (128-byte) column blocks
  static constexpr int kQBytes = kAtBM * D * 2;
  static constexpr int kKBytes = kAtBN * D * 2;
  static constexpr int kVBytes = kAtBN * D * 2;
  static constexpr int kStages = NB == 3 ? 2 : 1;
  static constexpr int kOffK = kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffBar = kOffV + kStages * kVBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
  static constexpr int kTmemCols = NB == 3 ? 512 : 256;  // NB S / P buffers of 128 columns, O (D)
  static constexpr int kOCol = NB * kAtBN;
  static_assert(kOCol + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct AtParams {
  __half* out;
  float* lse;
  int64_t s_q, s_kv, n_heads, n_kv_heads, q_pos_offset;
  int n_qblocks;
  int causal;
  float c;       // scale * log2(e)
  unsigned int* err;
  unsigned long long limit_ns;
};

/// 2^x by the MUFU approximation (ex2.approx.ftz.f32, relative error ~2^-22;
/// results below 2^-126 flush to zero -- probabilities that small vanish in the
/// FP16 P tile anyway).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

/// Keys visible to query row `row` (global index), as the last visible index.
__device__ __forceinline__ int64_t at_last_key(const AtParams& p, int64_t row) {
  int64_t lim = p.s_kv - 1;
  if (p.causal && p.q_pos_offset + row < lim) lim = p.q_pos_offset + row;
  return lim;
}

template <int D, int NS, int NB>
__global__ void __launch_bounds__(at_threads(NS), NB == 3 ? 1 : 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AtParams p) {
  using Cfg = AtCfg<D, NB>;
  constexpr int ST = Cfg::kStages;
  static_assert(NB == 1 || NB == 3, "one or three S / P buffers");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + Cfg::kOffK;
  uint8_t* sV = smem + Cfg::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bars;          // 1
  uint64_t* k_full = bars + 1;      // ST
  uint64_t* k_empty = k_full + ST;  // ST
  uint64_t* v_full = k_empty + ST;  // ST
  uint64_t* v_empty = v_full + ST;  // ST
  uint64_t* s_full = v_empty + ST;  // NB: S(j) in buffer j % NB complete
  uint64_t* p_full = s_full + 3;    // NB: P(j) written over it
  uint64_t* o_done = p_full + 3;    // NB: PV(j) complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 3);
  static_assert(kAtBN % (32 * NS) == 0 && D % (32 * NS) == 0, "column groups of 32");
  __shared__ float s_mx[2][NS][kAtBM];  // per-row exchange of the column groups' maxima
  __shared__ float s_lx[NS][kAtBM];     // ... and of their sums, at the end
  // One exchange barrier per lane quarter and tile parity, one for the sums:
  // mbarriers, so that every wait is bounded.
  __shared__ uint64_t xbar[2][4], lbar[4];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Heaviest q-blocks (most keys under the causal mask) first.
  const int qb = p.n_qblocks - 1 - static_cast<int>(blockIdx.x / p.n_heads);
  const int h = static_cast<int>(blockIdx.x % p.n_heads);
  const int hk = static_cast<int>(h / (p.n_heads / p.n_kv_heads));
  const int64_t q0 = static_cast<int64_t>(qb) * kAtBM;
  const int64_t last_row = (q0 + kAtBM - 1 < p.s_q - 1) ? q0 + kAtBM - 1 : p.s_q - 1;
  const int ntiles = static_cast<int>(at_last_key(p, last_row) / kAtBN) + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128 * NS);
      mbar_init(&o_done[b], 1);
    }
    for (int q = 0; q < 4; ++q) {
      mbar_init(&xbar[0][q], 32 * NS);
      mbar_init(&xbar[1][q], 32 * NS);
      mbar_init(&lbar[q], 32 * NS);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
#pragma unroll
      for (int dh = 0; dh < Cfg::kDH; ++dh)
        tma_load_3d(sQ + dh * 16384, &tmQ, q_full, dh * 64, h, static_cast<int32_t>(q0));
      int kn = 0, vn = 0;  // K / V tiles issued
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % ST;
        const uint32_t ph = (j / ST) & 1u;
        const int32_t j0 = j * kAtBN;
        if (!mbar_wait(&k_empty[s], ph ^ 1u, p.limit_ns, p.err)) break;
        mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
#pragma unroll
        for (int dh = 0; dh < Cfg::kDH; ++dh)
          tma_load_3d(sK + s * Cfg::kKBytes + dh * 16384, &tmK, &k_full[s], dh * 64, j0, hk);
        ++kn;
        if (!mbar_wait(&v_empty[s], ph ^ 1u, p.limit_ns, p.err)) break;
        mbar_arrive_expect_tx(&v_full[s], Cfg::kVBytes);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
#pragma unroll
          for (int dh = 0; dh < Cfg::kDH; ++dh)
            tma_load_3d(sV + s * Cfg::kVBytes + kh * (Cfg::kDH * 8192) + dh * 8192, &tmV,
                        &v_full[s], dh * 64, j0 + kh * 64, hk);
        }
        ++vn;
      }
      // No copy may still be writing shared memory when the CTA leaves: wait
      // (bounded) for the last loads issued into each ring stage.  On the normal
      // path these phases have long completed.
      mbar_wait(q_full, 0, p.limit_ns, p.err);
      for (int j = (kn > ST ? kn - ST : 0); j < kn; ++j)
        mbar_wait(&k_full[j % ST], (j / ST) & 1u, p.limit_ns, p.err);
      for (int j = (vn > ST ? vn - ST : 0); j < vn; ++j)
        mbar_wait(&v_full[j % ST], (j / ST) & 1u, p.limit_ns, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_f16(128, kAtBN, false, false, false);
      constexpr uint32_t kIdescO = umma_idesc_f16(128, D, false, false, true);
      const uint32_t tO = tmem_base + Cfg::kOCol;
      bool ok = mbar_wait(q_full, 0, p.limit_ns, p.err);
      const uint32_t q_addr = smem_u32(sQ);
      auto pv = [&](int i) {  // O += P[i] V[i], P[i] in TMEM over S[i]
        const int b = i % NB;
        const int s = i % ST;
        if (!mbar_wait(&p_full[b], (i / NB) & 1u, p.limit_ns, p.err)) return false;
        if (!mbar_wait(&v_full[s], (i / ST) & 1u, p.limit_ns, p.err)) return false;
        tc_fence_after();
        const uint32_t pa = tmem_base + b * kAtBN;
        const uint32_t va = smem_u32(sV + s * Cfg::kVBytes);
#pragma unroll
        for (int kk = 0; kk < kAtBN / 16; ++kk) {
          const uint64_t bdesc =
              umma_desc_sw128(va + (kk >> 2) * (Cfg::kDH * 8192) + (kk & 3) * 2048, 8192, 1024);
          umma_f16_ts(tO, pa + kk * 8, bdesc, kIdescO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[s]);
        umma_commit(&o_done[b]);
        return true;
      };
      int last_s = -1, last_pv = -1;  // last S / PV products issued
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j % ST;
        const int b = j % NB;
        if (!mbar_wait(&k_full[s], (j / ST) & 1u, p.limit_ns, p.err)) {
          ok = false;
          break;
        }
        if (NB == 1 && j >= 1) {  // one buffer: PV(j-1) reads it before S(j) overwrites
          if (pv(j - 1)) last_pv = j - 1;
          else {
            ok = false;
            break;
          }
        }
        // Buffer b last held P(j-NB): its PV product must have read it.
        if (j >= NB && !mbar_wait(&o_done[b], ((j - NB) / NB) & 1u, p.limit_ns, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + s * Cfg::kKBytes);
        const uint32_t tS = tmem_base + b * kAtBN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(q_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(ka + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          umma_f16(tS, adesc, bdesc, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[b]);
        last_s = j;
        if (NB > 1 && j >= 1) {
          if (pv(j - 1)) last_pv = j - 1;
          else ok = false;
        }
      }
      if (ok && pv(ntiles - 1)) last_pv = ntiles - 1;
      // No MMA may still use TMEM or shared memory when the CTA leaves: each
      // commit arrives once every earlier MMA completed, so wait (bounded) for
      // the later of the last two commits.
      if (last_pv >= 0 && last_pv >= last_s) {
        mbar_wait(&o_done[last_pv % NB], (last_pv / NB) & 1u, p.limit_ns, p.err);
      } else if (last_s >= 0) {
        mbar_wait(&s_full[last_s % NB], (last_s / NB) & 1u, p.limit_ns, p.err);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    // NS warps share each TMEM lane quarter: warp w reads lanes 32*(w%4)..+31
    // (its rows) and column group cg = (w-2)/4 of them -- CW keys of S and OW
    // columns of O.  The row max is combined across the NS threads of a row
    // through shared memory (one named barrier per lane quarter); the sums l
    // stay per thread until the end.
    constexpr int CW = kAtBN / NS;  // keys of S per thread
    constexpr int OW = D / NS;      // columns of O per thread
    const int q4 = warp & 3;
    const int cg = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;  // this thread's row of the tile (TMEM lane)
    const int64_t row = q0 + r;
    const int64_t lim = at_last_key(p, row);
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t tO = tmem_base + lane_base + Cfg::kOCol + cg * OW;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1;   // parity of the max exchange
      const int b3 = j % NB;  // S / P buffer
      bool w = mbar_wait_sleepy(&s_full[b3], (j / NB) & 1u, p.limit_ns, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[CW / 32][32];
      const uint32_t tS = tmem_base + lane_base + b3 * kAtBN + cg * CW;
#pragma unroll
      for (int c = 0; c < CW / 32; ++c) tmem_ld_32x32b_x32(tS + c * 32, sv[c]);
      tmem_wait_ld();
      const int64_t k0 = static_cast<int64_t>(j) * kAtBN + cg * CW;  // first key of this thread
      const bool full = k0 + CW - 1 <= lim;  // none of this thread's keys is masked
      // Raw scores: the scale c > 0 is folded into the exponent below, so the
      // row max is taken on S itself (c * max S = max c S).
      float mt0 = -INFINITY, mt1 = -INFINITY;
      if (!full) {
#pragma unroll
        for (int c = 0; c < CW / 32; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (k0 + c * 32 + e > lim) sv[c][e] = __float_as_uint(-INFINITY);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < CW / 32; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          mt0 = fmaxf(mt0, __uint_as_float(sv[c][e]));
          mt1 = fmaxf(mt1, __uint_as_float(sv[c][e + 1]));
        }
      }
      float mt = fmaxf(mt0, mt1);
      if constexpr (NS > 1) {
        s_mx[b][cg][r] = mt;
        mbar_arrive(&xbar[b][q4]);
        w = mbar_wait_sleepy(&xbar[b][q4], (j >> 1) & 1u, p.limit_ns, p.err);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int g = 0; g < NS; ++g) mt = fmaxf(mt, s_mx[b][g][r]);
      }
      mt *= p.c;  // base-2 domain
      // Lazy rescaling: the row keeps its reference max m until a tile's max
      // exceeds it by more than kAtRescale (base 2), so P = exp2(S*c - m) stays
      // below 2^kAtRescale (exact enough in FP16) and O needs rescaling only on
      // such jumps.  The final O / l and lse = m ln 2 + ln l do not depend on
      // which reference was used.
      const bool first = (m == -INFINITY);
      const bool rescale = !first && mt > m + kAtRescale;
      const float m_new = (first || rescale) ? fmaxf(m, mt) : m;
      // With no visible key yet the row keeps m = -inf and P = 0.
      const float base = (m_new == -INFINITY) ? 0.0f : m_new;
      const float alpha = ex2_fast(m - base);  // m = -inf -> 0; no rescale -> 1
      float ls0 = 0.0f, ls1 = 0.0f;
      uint32_t pk[CW / 32][16];  // P as FP16 pairs
#pragma unroll
      for (int c = 0; c < CW / 32; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = ex2_fast(fmaf(__uint_as_float(sv[c][e]), p.c, -base));
          const float p1 = ex2_fast(fmaf(__uint_as_float(sv[c][e + 1]), p.c, -base));
          ls0 += p0;
          ls1 += p1;
          __half2 hv = __floats2half2_rn(p0, p1);
          pk[c][e >> 1] = *reinterpret_cast<uint32_t*>(&hv);
        }
      }
      l = l * alpha + (ls0 + ls1);
      m = m_new;
      // P(j) goes over this thread's row of S(j) in TMEM: keys [cg*CW, +CW) as
      // CW/2 packed columns from column cg*CW/2.  The row's other threads have
      // already read their S (they arrived at the max exchange after
      // tcgen05.wait::ld), so no score is overwritten before it is read.
      const uint32_t tP = tmem_base + lane_base + b3 * kAtBN + cg * (CW / 2);
#pragma unroll
      for (int c = 0; c < CW / 32; ++c) tmem_st_32x32b_x16(tP + c * 16, pk[c]);
      // O may be rescaled only once PV(j-1) completed (PV(j) waits for p_full).
      const bool any_rescale = __any_sync(0xffffffffu, rescale);
      if (any_rescale) {
        if (j >= 1) {
          w = mbar_wait_sleepy(&o_done[(j - 1) % NB], ((j - 1) / NB) & 1u, p.limit_ns, p.err);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < OW / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tO + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st_32x32b_x32(tO + c * 32, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[b3]);
    }
    // Row sums: the NS partial sums of a row, added in column-group order.
    if (NS > 1 && ok) {
      s_lx[cg][r] = l;
      mbar_arrive(&lbar[q4]);
      ok = __all_sync(0xffffffffu, mbar_wait_sleepy(&lbar[q4], 0, p.limit_ns, p.err));
      l = 0.0f;
#pragma unroll
      for (int g = 0; g < NS; ++g) l += s_lx[g][r];
    }
    if (ok) {
      const int last = ntiles - 1;
      const bool w = mbar_wait_sleepy(&o_done[last % NB], (last / NB) & 1u, p.limit_ns, p.err);
      if (__all_sync(0xffffffffu, w)) {
        tc_fence_after();
        const float inv = 1.0f / l;
        __half* orow = p.out + (row * p.n_heads + h) * D + cg * OW;
#pragma unroll 1
        for (int c = 0; c < OW / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tO + c * 32, ov);
          tmem_wait_ld();
          if (row < p.s_q) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              __half2 h0 = __floats2half2_rn(__uint_as_float(ov[8 * g]) * inv,
                                             __uint_as_float(ov[8 * g + 1]) * inv);
              __half2 h1 = __floats2half2_rn(__uint_as_float(ov[8 * g + 2]) * inv,
                                             __uint_as_float(ov[8 * g + 3]) * inv);
              __half2 h2 = __floats2half2_rn(__uint_as_float(ov[8 * g + 4]) * inv,
                                             __uint_as_float(ov[8 * g + 5]) * inv);
              __half2 h3 = __floats2half2_rn(__uint_as_float(ov[8 * g + 6]) * inv,
                                             __uint_as_float(ov[8 * g + 7]) * inv);
              dst[g] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                                  *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
            }
          }
        }
        if (cg == 0 && row < p.s_q && p.lse != nullptr)
          p.lse[row * p.n_heads + h] = m * 0.69314718055994531f + logf(l);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <int D, int NS, int NB>
int launch_attn_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const AtParams& p, cudaStream_t stream) {
  using Cfg = AtCfg<D, NB>;
  auto kern = attn_tc_kernel<D, NS, NB>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load() & bit) == 0) {
    B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::kSmemBytes));
    configured.fetch_or(bit);
  }
  const unsigned grid = static_cast<unsigned>(static_cast<int64_t>(p.n_qblocks) * p.n_heads);
  B200_CUDA(launch_pdl(kern, dim3(grid), dim3(at_threads(NS)), Cfg::kSmemBytes, stream, tq, tk, tv, p));
  return ENGINE_OK;
}

// ---------------------------------------------------------------- decode
//
// attention_decode (one query position, non-causal) on tcgen05.  A CTA takes
// one KV head and one split of its keys, in blocks of 128 keys, and serves the
// G <= 16 query heads of that KV group together.  The products are formed
// transposed, so that the 128 keys of a block (and later the d = 128 output
// elements) fill the MMA's M = 128 rows:
//   S^T[key, h] = K[key, :] . q[h, :]      A = K block (TMA, K-major), B = q^T
//                                           (16 rows: the group's heads, the
//                                           rows past them never used), N = 16
//   O^T[e, h] += sum_key V[key, e] P[h, key]  A = V block as an MN-major operand
//                                           (TMA), B = P^T written to shared
//                                           memory by the softmax, N = 16
// Warp 0 issues the TMA loads (q once, K / V blocks into nst-stage rings),
// warp 1 owns TMEM (two 16-column S^T buffers and the O^T accumulator) and
// issues the MMAs, warps 2-5 run the softmax: thread t holds key t of the
// block (TMEM lane t) for all heads, takes each head's block maximum across
// the 128 threads (warp shuffles, then a bounded mbarrier exchange), keeps the
// running max m_h (base 2) with the lazy 2^8 rescaling of the prefill kernel,
// writes P = exp2(S c - m_h) as FP16 into the swizzled P^T tile and keeps its
// own partial sums l_h.  At the end thread e holds O^T[e, :] (TMEM lane e).  A
// single split writes out and lse directly.  Otherwise the R <= 16 splits of a
// KV head form one thread-block cluster: each CTA parks its (m, l, O) in its
// own shared memory, and after a cluster barrier the CTAs combine them through
// distributed shared memory (rank order, base 2) and write out and lse -- no
// workspace and no second kernel.
constexpr int kDtBlock = 128;  // keys per block
constexpr int kDtN = 16;       // MMA N: query heads of one KV group, padded
constexpr int kDtThreads = 192;

struct DtParams {
  __half* out;
  float* lse;
  float* ws;      // kDtWs: [n_heads][splits][D + 2], m (natural log), l, O
  int64_t s_kv, n_heads, group;
  int64_t chunk;  // keys per split (a multiple of kDtBlock)
  int splits;     // CTAs per KV head: the cluster size when > 1
  int nst;        // K / V ring stages
  float c;        // scale * log2(e)
  unsigned int* err;
  unsigned long long limit_ns;
};

template <int D>
struct DtCfg {
  static constexpr int kQBytes = kDtN * D * 2;          // 4 KB
  static constexpr int kKBytes = kDtBlock * D * 2;      // 32 KB
  static constexpr int kPBytes = kDtN * kDtBlock * 2;   // 4 KB
  static constexpr int smem(int nst) { return kQBytes + 2 * kPBytes + nst * 2 * kKBytes + 256 + 1024; }
};

// MODE: kDtFinal (one split: out and lse), kDtWs (splits to the workspace for
// attn_merge_kernel), kDtCluster (splits merged inside the cluster).
constexpr int kDtFinal = 0, kDtWs = 1, kDtCluster = 2;

template <int D, int MODE>
__global__ void __launch_bounds__(kDtThreads)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const DtParams p) {
  using Cfg = DtCfg<D>;
  static_assert(D == 128, "the O^T product uses M = d = 128");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int nst = p.nst;
  uint8_t* sQ = smem;
  uint8_t* sP = smem + Cfg::kQBytes;                    // two P^T tiles
  uint8_t* sK = sP + 2 * Cfg::kPBytes;                  // nst stages
  uint8_t* sV = sK + nst * Cfg::kKBytes;                // nst stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + nst * Cfg::kKBytes);
  uint64_t* q_full = bars;           // 1
  uint64_t* k_full = bars + 1;       // 2 (nst <= 2)
  uint64_t* k_empty = k_full + 2;
  uint64_t* v_full = k_empty + 2;
  uint64_t* v_empty = v_full + 2;
  uint64_t* s_full = v_empty + 2;    // 2
  uint64_t* p_full = s_full + 2;     // 2
  uint64_t* o_done = p_full + 2;     // 2
  uint64_t* xbar = o_done + 2;       // 2: the block-max exchange, by parity
  uint64_t* lbar = xbar + 2;         // 1: the final sums
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lbar + 1);
  __shared__ float s_mx[2][4][kDtN];
  __shared__ float s_l[4][kDtN];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int hk = blockIdx.y;
  const int64_t h0 = static_cast<int64_t>(hk) * p.group;  // first query head of the group
  const int G = static_cast<int>(p.group);
  const int64_t j0 = static_cast<int64_t>(split) * p.chunk;
  const int64_t j1 = (j0 + p.chunk < p.s_kv) ? j0 + p.chunk : p.s_kv;
  const int nblk = j1 > j0 ? static_cast<int>((j1 - j0 + kDtBlock - 1) / kDtBlock) : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_done[s], 1);
      mbar_init(&xbar[s], 128);
    }
    mbar_init(lbar, 128);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  if (warp >= 2) {  // the P^T rows past the group's heads stay zero
    for (int i = threadIdx.x - 64; i < 2 * Cfg::kPBytes / 16; i += 128)
      reinterpret_cast<uint4*>(sP)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
#pragma unroll
      for (int dh = 0; dh < D / 64; ++dh)
        tma_load_2d(sQ + dh * (kDtN * 128), &tmQ, q_full, dh * 64, static_cast<int32_t>(h0));
      int kn = 0, vn = 0;
      for (int b = 0; b < nblk; ++b) {
        const int s = b % nst;
        const uint32_t ph = (b / nst) & 1u;
        const int32_t jb = static_cast<int32_t>(j0 + static_cast<int64_t>(b) * kDtBlock);
        if (!mbar_wait(&k_empty[s], ph ^ 1u, p.limit_ns, p.err)) break;
        mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
#pragma unroll
        for (int dh = 0; dh < D / 64; ++dh)
          tma_load_3d(sK + s * Cfg::kKBytes + dh * 16384, &tmK, &k_full[s], dh * 64, jb, hk);
        ++kn;
        if (!mbar_wait(&v_empty[s], ph ^ 1u, p.limit_ns, p.err)) break;
        mbar_arrive_expect_tx(&v_full[s], Cfg::kKBytes);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
#pragma unroll
          for (int dh = 0; dh < D / 64; ++dh)
            tma_load_3d(sV + s * Cfg::kKBytes + kh * (D / 64) * 8192 + dh * 8192, &tmV, &v_full[s],
                        dh * 64, jb + kh * 64, hk);
        }
        ++vn;
      }
      mbar_wait(q_full, 0, p.limit_ns, p.err);
      for (int b = (kn > nst ? kn - nst : 0); b < kn; ++b)
        mbar_wait(&k_full[b % nst], (b / nst) & 1u, p.limit_ns, p.err);
      for (int b = (vn > nst ? vn - nst : 0); b < vn; ++b)
        mbar_wait(&v_full[b % nst], (b / nst) & 1u, p.limit_ns, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_f16(128, kDtN, false, false, false);
      constexpr uint32_t kIdescO = umma_idesc_f16(128, kDtN, false, true, false);
      const uint32_t tO = tmem_base + 32;
      bool ok = mbar_wait(q_full, 0, p.limit_ns, p.err);
      const uint32_t q_addr = smem_u32(sQ);
      int last_s = -1, last_pv = -1;
      auto pv = [&](int i) {  // O^T += V[i]^T P[i]^T
        const int s = i % nst;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1u, p.limit_ns, p.err)) return false;
        if (!mbar_wait(&v_full[s], (i / nst) & 1u, p.limit_ns, p.err)) return false;
        tc_fence_after();
        const uint32_t va = smem_u32(sV + s * Cfg::kKBytes);
        const uint32_t pa = smem_u32(sP + (i & 1) * Cfg::kPBytes);
#pragma unroll
        for (int kk = 0; kk < kDtBlock / 16; ++kk) {
          const uint64_t adesc =
              umma_desc_sw128(va + (kk >> 2) * ((D / 64) * 8192) + (kk & 3) * 2048, 8192, 1024);
          const uint64_t bdesc = umma_desc_sw128(pa + (kk >> 2) * (kDtN * 128) + (kk & 3) * 32, 16, 1024);
          umma_f16(tO, adesc, bdesc, kIdescO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[s]);
        umma_commit(&o_done[i & 1]);
        last_pv = i;
        return true;
      };
      for (int b = 0; ok && b < nblk; ++b) {
        const int s = b % nst;
        if (!mbar_wait(&k_full[s], (b / nst) & 1u, p.limit_ns, p.err)) break;
        // S^T buffer b & 1 was last read by the softmax of block b - 2, which
        // finished before P(b-2) was released: PV(b-2) has been issued after it.
        if (b >= 2 && !mbar_wait(&p_full[b & 1], ((b - 2) >> 1) & 1u, p.limit_ns, p.err)) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + s * Cfg::kKBytes);
        const uint32_t tS = tmem_base + (b & 1) * kDtN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(ka + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(q_addr + (kk >> 2) * (kDtN * 128) + (kk & 3) * 32, 16, 1024);
          umma_f16(tS, adesc, bdesc, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[b & 1]);
        last_s = b;
        if (b >= 1 && !pv(b - 1)) ok = false;
      }
      if (ok && nblk > 0) pv(nblk - 1);
      if (last_pv >= 0 && last_pv >= last_s) {
        mbar_wait(&o_done[last_pv & 1], (last_pv >> 1) & 1u, p.limit_ns, p.err);
      } else if (last_s >= 0) {
        mbar_wait(&s_full[last_s & 1], (last_s >> 1) & 1u, p.limit_ns, p.err);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int t = q4 * 32 + lane;  // key of the block / output element
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    float m[kDtN], l[kDtN];
#pragma unroll
    for (int h = 0; h < kDtN; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.0f;
    }
    bool ok = true;
    for (int b = 0; b < nblk; ++b) {
      const int bb = b & 1;
      bool w = mbar_wait_sleepy(&s_full[bb], (b >> 1) & 1u, p.limit_ns, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[kDtN];
      tmem_ld_32x32b_x16(tmem_base + lane_base + bb * kDtN, sv);
      tmem_wait_ld();
      const int64_t key = j0 + static_cast<int64_t>(b) * kDtBlock + t;
      const bool valid = key < j1;
      float x[kDtN], mx[kDtN];
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        x[h] = valid ? __uint_as_float(sv[h]) : -INFINITY;
        mx[h] = x[h];
      }
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        if (h < G) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], o));
        }
      }
      if (lane < kDtN) {
        float v = mx[0];
#pragma unroll
        for (int h = 1; h < kDtN; ++h) v = (lane == h) ? mx[h] : v;
        s_mx[bb][q4][lane] = v;
      }
      mbar_arrive(&xbar[bb]);
      w = mbar_wait_sleepy(&xbar[bb], (b >> 1) & 1u, p.limit_ns, p.err);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      // P^T tile bb is free once PV(b-2) completed; O may be rescaled only once
      // PV(b-1) completed (PV(b) waits for this block's p_full).
      bool rescale_any = false;
      float alpha[kDtN], base[kDtN];
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        const float bm = fmaxf(fmaxf(s_mx[bb][0][h], s_mx[bb][1][h]),
                               fmaxf(s_mx[bb][2][h], s_mx[bb][3][h])) * p.c;
        const bool first = (m[h] == -INFINITY);
        const bool rs = !first && bm > m[h] + kAtRescale;
        const float mn = (first || rs) ? fmaxf(m[h], bm) : m[h];
        base[h] = (mn == -INFINITY) ? 0.0f : mn;
        alpha[h] = ex2_fast(m[h] - base[h]);
        rescale_any |= (h < G) && rs;
        m[h] = mn;
      }
      const int dep = rescale_any ? b - 1 : b - 2;
      if (dep >= 0) {
        w = mbar_wait_sleepy(&o_done[dep & 1], (dep >> 1) & 1u, p.limit_ns, p.err);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
      }
      // P^T[h][t]: row h (128 bytes per 64 keys), 16-byte chunk (t % 64) / 8
      // swizzled by h % 8, element t % 8.
      uint8_t* pt = sP + bb * Cfg::kPBytes + (t >> 6) * (kDtN * 128);
      const int chunk = (t & 63) >> 3;
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        if (h < G) {
          const float pv = ex2_fast(fmaf(x[h], p.c, -base[h]));
          l[h] = l[h] * alpha[h] + pv;
          *reinterpret_cast<__half*>(pt + h * 128 + ((chunk ^ (h & 7)) << 4) + (t & 7) * 2) =
              __float2half_rn(pv);
        }
      }
      if (rescale_any) {  // thread t owns output element t of every head (TMEM lane t)
        tc_fence_after();
        uint32_t ov[kDtN];
        tmem_ld_32x32b_x16(tmem_base + lane_base + 32, ov);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < kDtN; ++h) ov[h] = __float_as_uint(__uint_as_float(ov[h]) * alpha[h]);
        tmem_st_32x32b_x16(tmem_base + lane_base + 32, ov);
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[bb]);
    }
    // Per-head sums over the 128 threads, then the output.
    if (ok) {
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        if (h < G) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) l[h] += __shfl_xor_sync(0xffffffffu, l[h], o);
        }
      }
      if (lane < kDtN) {
        float v = l[0];
#pragma unroll
        for (int h = 1; h < kDtN; ++h) v = (lane == h) ? l[h] : v;
        s_l[q4][lane] = v;
      }
      mbar_arrive(lbar);
      ok = __all_sync(0xffffffffu, mbar_wait_sleepy(lbar, 0, p.limit_ns, p.err));
    }
    if (ok && nblk > 0) {
      const int last = nblk - 1;
      ok = __all_sync(0xffffffffu,
                      mbar_wait_sleepy(&o_done[last & 1], (last >> 1) & 1u, p.limit_ns, p.err));
    }
    if (ok) {
      uint32_t ov[kDtN];
      if (nblk > 0) {
        tc_fence_after();
        tmem_ld_32x32b_x16(tmem_base + lane_base + 32, ov);
        tmem_wait_ld();
      }
#pragma unroll
      for (int h = 0; h < kDtN; ++h) {
        if (h >= G) continue;
        const float L = (s_l[0][h] + s_l[1][h]) + (s_l[2][h] + s_l[3][h]);
        const float o = nblk > 0 ? __uint_as_float(ov[h]) : 0.0f;
        const int64_t row = h0 + h;
        const float mnat = (nblk > 0 && m[h] != -INFINITY) ? m[h] * 0.69314718055994531f : -INFINITY;
        if constexpr (MODE == kDtFinal) {
          p.out[row * D + t] = __float2half_rn(L > 0.0f ? o / L : 0.0f);
          if (t == 0 && p.lse != nullptr) p.lse[row] = L > 0.0f ? mnat + logf(L) : -INFINITY;
        } else if constexpr (MODE == kDtWs) {
          float* wsr = p.ws + (row * p.splits + split) * (D + 2);
          if (t == 0) {
            wsr[0] = mnat;
            wsr[1] = L;
          }
          wsr[2 + t] = o;
        } else {
          // The partial for the cluster merge: O[h][e], then m[h] (base 2), l[h].
          float* part = reinterpret_cast<float*>(sK);
          part[h * D + t] = o;
          if (t == 0) {
            part[kDtN * D + h] = (nblk > 0) ? m[h] : -INFINITY;
            part[kDtN * D + kDtN + h] = L;
          }
        }
      }
    }
  }
  if constexpr (MODE == kDtCluster) {
    // Every thread of every CTA reaches both cluster barriers (no early exit on
    // any path; the waits above are bounded).  The first makes each CTA's
    // partial visible cluster-wide; the second keeps every CTA resident until
    // its partial has been read.
    __syncwarp();
    cluster_sync_all();
    if (warp >= 2) {
      const int t = (warp & 3) * 32 + lane;
      const int R = p.splits;
      const uint32_t rank = cluster_ctarank();
      const uint32_t part = smem_u32(sK);
      for (int idx = static_cast<int>(rank) * 128 + t; idx < G * D; idx += R * 128) {
        const int h = idx / D, e = idx % D;
        float M = -INFINITY;
        for (int q = 0; q < R; ++q)
          M = fmaxf(M, ld_dsmem_f32(mapa_shared(part + 4u * (kDtN * D + h), q)));
        float Ls = 0.0f, Os = 0.0f;
        for (int q = 0; q < R; ++q) {
          const float mq = ld_dsmem_f32(mapa_shared(part + 4u * (kDtN * D + h), q));
          const float wq = (mq == -INFINITY) ? 0.0f : ex2_fast(mq - M);
          Ls = fmaf(ld_dsmem_f32(mapa_shared(part + 4u * (kDtN * D + kDtN + h), q)), wq, Ls);
          Os = fmaf(ld_dsmem_f32(mapa_shared(part + 4u * (h * D + e), q)), wq, Os);
        }
        const int64_t row = h0 + h;
        p.out[row * D + e] = __float2half_rn(Ls > 0.0f ? Os / Ls : 0.0f);
        if (e == 0 && p.lse != nullptr)
          p.lse[row] = Ls > 0.0f ? M * 0.69314718055994531f + logf(Ls) : -INFINITY;
      }
    }
    cluster_sync_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 64);
  }
}

template <int D, int MODE>
cudaLaunchConfig_t decode_tc_config(const DtParams& p, unsigned n_kv_heads, cudaStream_t stream,
                                    cudaLaunchAttribute (&attr)[2]) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.splits), n_kv_heads);
  cfg.blockDim = dim3(kDtThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(DtCfg<D>::smem(p.nst));
  cfg.stream = stream;
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  if (pdl_enabled()) ++n;
  if (MODE == kDtCluster) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(p.splits);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cfg;
}

template <int D, int MODE>
int configure_decode_tc() {
  auto kern = attn_decode_tc_kernel<D, MODE>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load() & bit) == 0) {
    B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   DtCfg<D>::smem(2)));
    configured.fetch_or(bit);
  }
  return ENGINE_OK;
}

}  // namespace

int attention_prefill_tc(const __half* q, const __half* k, const __half* v, __half* out,
                         int64_t s_q, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads, int64_t d,
                         int64_t kv_head_stride, float scale, int64_t q_pos_offset, bool causal,
                         float* lse, cudaStream_t stream) {
  if ((d != 64 && d != 128) || !(scale > 0.0f) || kv_head_stride % 8 != 0 ||
      s_q > (int64_t{1} << 31) ||
      (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) % 16 != 0 ||
      s_kv > (int64_t{1} << 31) || n_heads > 65535 || n_kv_heads > 65535)
    return ENGINE_ERR_UNSUPPORTED;
  const uint64_t qd[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(n_heads),
                          static_cast<uint64_t>(s_q)};
  const uint64_t qs[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(n_heads * d)};
  const uint32_t qbox[3] = {64, 1, kAtBM};
  const uint64_t kd[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(s_kv),
                          static_cast<uint64_t>(n_kv_heads)};
  const uint64_t ks[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(kv_head_stride)};
  const uint32_t kbox[3] = {64, kAtBN, 1};
  const uint32_t vbox[3] = {64, 64, 1};
  CUtensorMap tq, tk, tv;
  if (!make_tmap_3d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, qd, qs, qbox) ||
      !make_tmap_3d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kd, ks, kbox) ||
      !make_tmap_3d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kd, ks, vbox))
    return ENGINE_ERR_UNSUPPORTED;
  AtParams p{};
  p.out = out;
  p.lse = lse;
  p.s_q = s_q;
  p.s_kv = s_kv;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.q_pos_offset = q_pos_offset;
  p.n_qblocks = static_cast<int>((s_q + kAtBM - 1) / kAtBM);
  p.causal = causal ? 1 : 0;
  p.c = scale * 1.4426950408889634f;
  p.err = device_error_word();
  p.limit_ns = wait_limit_ns();
  const int rc = (d == 64) ? launch_attn_tc<64, kAtSplit64, kAtBufs>(tq, tk, tv, p, stream)
                           : launch_attn_tc<128, kAtSplit128, kAtBufs>(tq, tk, tv, p, stream);
  if (rc != ENGINE_OK) return rc;
  return check_launch("attention_prefill");
}

}  // namespace b200

namespace b200 {

// Split plan: about two CTAs per SM over all KV heads (single-stage K / V
// rings, 79 KB of shared memory each), whole 128-key blocks per split.  One
// split per head writes out directly; up to 8 merge inside a cluster
// (portable size); more go through the workspace and attn_merge_kernel.
// (Clusters of 16 were measured: a GPC rarely has 16 free SMs, so they could
// not all be resident.)
struct DtPlan {
  int splits;
  int64_t chunk;
  int nst;  // K / V ring stages
};

DtPlan decode_tc_plan(int64_t s_kv, int64_t n_kv_heads) {
  const int64_t nblocks = (s_kv + kDtBlock - 1) / kDtBlock;
  const int64_t want = std::max<int64_t>(1, (2 * static_cast<int64_t>(sm_count())) / n_kv_heads);
  int64_t bpc = (nblocks + want - 1) / want;  // blocks per split
  int64_t splits = (nblocks + bpc - 1) / bpc;
  int nst = 1;
  // 9-16 key blocks per KV head: a cluster of at most 8 CTAs with two blocks
  // each and a two-stage K / V ring, merged in the cluster, instead of one-block
  // splits merged through the workspace by a second kernel (B200, 32 query / 8 KV
  // heads, 2048 keys: 10.2 -> 8.9 us; at 4096 keys four blocks per CTA were no
  // faster than the workspace merge, at 8192 slower).
  if (splits > 8 && nblocks <= 16) {
    bpc = (nblocks + 7) / 8;
    splits = (nblocks + bpc - 1) / bpc;
    nst = 2;
  }
  return {static_cast<int>(splits), bpc * kDtBlock, nst};
}

int attention_decode_tc_splits(int64_t s_kv, int64_t n_kv_heads, int64_t* chunk) {
  const DtPlan pl = decode_tc_plan(s_kv, n_kv_heads);
  *chunk = pl.chunk;
  return pl.splits <= 8 ? 0 : pl.splits;  // 0: no workspace
}

int attention_decode_tc(const __half* q, const __half* k, const __half* v, __half* out, float* lse,
                        float* ws, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads, int64_t d,
                        int64_t kv_head_stride, float scale, cudaStream_t stream) {
  const int64_t group = n_kv_heads > 0 ? n_heads / n_kv_heads : 0;
  if (d != 128 || group < 1 || group > kDtN || !(scale > 0.0f) || kv_head_stride % 8 != 0 ||
      s_kv < 1 || s_kv > (int64_t{1} << 31) || n_kv_heads > 65535 ||
      (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) % 16 != 0)
    return ENGINE_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  const uint64_t kd[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(s_kv),
                          static_cast<uint64_t>(n_kv_heads)};
  const uint64_t ks[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(kv_head_stride)};
  const uint32_t kbox[3] = {64, kDtBlock, 1};
  const uint32_t vbox[3] = {64, 64, 1};
  if (!make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(n_heads),
                    static_cast<uint64_t>(d), static_cast<uint64_t>(d), kDtN, 64) ||
      !make_tmap_3d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kd, ks, kbox) ||
      !make_tmap_3d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kd, ks, vbox))
    return ENGINE_ERR_UNSUPPORTED;
  DtParams p{};
  p.out = out;
  p.lse = lse;
  p.s_kv = s_kv;
  p.n_heads = n_heads;
  p.group = group;
  p.c = scale * 1.4426950408889634f;
  p.err = device_error_word();
  p.limit_ns = wait_limit_ns();
  const DtPlan pl = decode_tc_plan(s_kv, n_kv_heads);
  const unsigned hk = static_cast<unsigned>(n_kv_heads);
  p.splits = pl.splits;
  p.chunk = pl.chunk;
  p.nst = pl.nst;
  cudaLaunchAttribute attr[2];
  if (pl.splits == 1) {
    const int rc = configure_decode_tc<128, kDtFinal>();
    if (rc != ENGINE_OK) return rc;
    cudaLaunchConfig_t cfg = decode_tc_config<128, kDtFinal>(p, hk, stream, attr);
    B200_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_tc_kernel<128, kDtFinal>, tq, tk, tv, p));
  } else if (pl.splits <= 8) {
    const int rc = configure_decode_tc<128, kDtCluster>();
    if (rc != ENGINE_OK) return rc;
    cudaLaunchConfig_t cfg = decode_tc_config<128, kDtCluster>(p, hk, stream, attr);
    B200_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_tc_kernel<128, kDtCluster>, tq, tk, tv, p));
  } else {
    if (ws == nullptr) return ENGINE_ERR_UNSUPPORTED;  // sized by attention_decode_tc_splits
    p.ws = ws;
    const int rc = configure_decode_tc<128, kDtWs>();
    if (rc != ENGINE_OK) return rc;
    cudaLaunchConfig_t cfg = decode_tc_config<128, kDtWs>(p, hk, stream, attr);
    B200_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_tc_kernel<128, kDtWs>, tq, tk, tv, p));
  }
  return check_launch("attention_decode");
}

}  // namespace b200
