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
#include <atomic>
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
