// attention.cu -- MHA / GQA attention: split-KV decode and a prefill baseline.
//
// Layouts and contract of the engine's launchers (include/engine/kernels.hpp:153
// attention_prefill, :191 attention_decode; kernels/attention_prefill.cu:329-360,
// kernels/attention_decode.cu:637-660): q / out [s_q][n_heads][d], k / v
// [n_kv_heads][kv_head_stride] with key j of a KV head at j * d, d = 64 or 128,
// query head h reading KV head h / (n_heads / n_kv_heads).  Query row i sees
// keys j <= q_pos_offset + i when causal, every key otherwise.
//
// Dispatch (run_attention and the two entry points at the end of this file):
// - attention_prefill from 16 query rows: the tcgen05 FlashAttention kernel in
//   attention_tc.cu;
// - attention_decode (and a one-row non-causal prefill) with head_dim 128, at
//   most 16 query heads per KV head and automatic splits: the tcgen05 decode
//   kernel in attention_tc.cu, its splits combined inside a thread-block
//   cluster (up to 8 key blocks of 128 per KV head) or by attn_merge_kernel;
// - other decode shapes and explicit split counts: attn_decode_bulk_kernel
//   below (K / V blocks by cp.async.bulk, CUDA-core arithmetic);
// - everything else (a few query rows, unaligned strides): attn_split_kernel,
//   the CUDA-core baseline.  A CTA takes one query position, up to four query
//   heads of one KV group and one split of the key range; its 4 warps stream
//   that KV head's K and V rows with 16-byte loads (d / 8 lanes per key row),
//   each lane group runs an FP32 online softmax over its keys, the CTA merges
//   its lane groups in fixed order through shared memory, and a single split
//   writes out (and lse) directly while more splits write (m, l, O) to a
//   workspace that attn_merge_kernel combines in split order.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace b200 {
namespace {

constexpr int kAttnWarps = 4;
// attention_prefill takes the tcgen05 kernel from this many query rows up; below
// it, the split kernel's per-position CTAs fill the GPU better.
constexpr int64_t kAttnTcMinRows = 16;

int env_flag(const char* name, int dflt) {
  const char* e = std::getenv(name);
  if (e == nullptr || e[0] == '\0') return dflt;
  return static_cast<int>(std::strtol(e, nullptr, 10));
}
constexpr int kAttnUnroll = 4;  // keys per lane group per step (loads issued first)

template <bool VEC>
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
  if constexpr (VEC) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = __half2float(p[i]);
  }
}

struct AttnArgs {
  const __half* q;
  const __half* k;
  const __half* v;
  __half* out;
  float* lse;
  float* ws;  // [s_q * n_heads][splits][d + 2]: m, l, O[d]
  int64_t s_q, s_kv, n_heads, n_kv_heads, kv_head_stride, q_pos_offset;
  float scale;
  int causal;
  int splits;
  int64_t chunk;  // keys per split
};

// grid: (splits, n_kv_heads * (group / GB), s_q); block: 128 threads.
template <int D, int GB, bool VEC, bool FINAL>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(const AttnArgs a) {
  constexpr int LPK = D / 8;               // lanes per key row
  constexpr int KPW = 32 / LPK;            // key rows per warp
  constexpr int NKG = kAttnWarps * KPW;    // lane groups per CTA
  __shared__ float s_m[NKG][GB], s_l[NKG][GB];
  __shared__ float s_o[NKG][GB][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % LPK;              // this lane's 8 elements: [8 sub, 8 sub + 8)
  const int kgw = lane / LPK;              // lane group within the warp
  const int kg = warp * KPW + kgw;         // lane group within the CTA
  const int64_t group = a.n_heads / a.n_kv_heads;
  const int64_t chunks_per_kv = group / GB;
  const int64_t h_kv = blockIdx.y / chunks_per_kv;
  const int64_t h0 = h_kv * group + (blockIdx.y % chunks_per_kv) * GB;  // first query head
  const int64_t i = blockIdx.z;                                         // query position
  const int split = blockIdx.x;
  pdl_trigger();
  pdl_wait();

  int64_t max_j = a.s_kv - 1;
  if (a.causal && a.q_pos_offset + i < max_j) max_j = a.q_pos_offset + i;
  const int64_t j0 = static_cast<int64_t>(split) * a.chunk;
  int64_t j1 = j0 + a.chunk;
  if (j1 > max_j + 1) j1 = max_j + 1;  // keys [j0, j1) of this split are visible

  float qf[GB][8];
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    load8<VEC>(a.q + ((i * a.n_heads) + h0 + g) * D + 8 * sub, qf[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[g][e] *= a.scale;
  }
  float m[GB], l[GB], o[GB][8];
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[g][e] = 0.0f;
  }
  const __half* kh = a.k + h_kv * a.kv_head_stride + 8 * sub;
  const __half* vh = a.v + h_kv * a.kv_head_stride + 8 * sub;
  // The loop bound is uniform across the warp (the shuffles below need every
  // lane); lane group kgw takes key jw + kgw + u * NKG.
  for (int64_t jw = j0 + static_cast<int64_t>(warp) * KPW; jw < j1;
       jw += static_cast<int64_t>(NKG) * kAttnUnroll) {
    const int64_t jb = jw + kgw;
    float kf[kAttnUnroll][8], vf[kAttnUnroll][8];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int64_t j = jb + static_cast<int64_t>(u) * NKG;
      if (j < j1) {
        load8<VEC>(kh + j * D, kf[u]);
        load8<VEC>(vh + j * D, vf[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int64_t j = jb + static_cast<int64_t>(u) * NKG;
      const bool valid = j < j1;  // uniform within a lane group
#pragma unroll
      for (int g = 0; g < GB; ++g) {
        float s = 0.0f;
        if (valid) {
#pragma unroll
          for (int e = 0; e < 8; ++e) s = fmaf(qf[g][e], kf[u][e], s);
        }
#pragma unroll
        for (int off = LPK / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (valid) {
          const float mn = fmaxf(m[g], s);
          const float alpha = expf(m[g] - mn);  // m = -inf first: alpha = 0
          const float p = expf(s - mn);
          l[g] = l[g] * alpha + p;
#pragma unroll
          for (int e = 0; e < 8; ++e) o[g][e] = fmaf(p, vf[u][e], o[g][e] * alpha);
          m[g] = mn;
        }
      }
    }
  }
  // merge the lane groups in fixed order
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    if (sub == 0) {
      s_m[kg][g] = m[g];
      s_l[kg][g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s_o[kg][g][8 * sub + e] = o[g][e];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < GB * D; t += blockDim.x) {
    const int g = t / D, d = t % D;
    float M = -INFINITY;
    for (int c = 0; c < NKG; ++c) M = fmaxf(M, s_m[c][g]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int c = 0; c < NKG; ++c) {
        if (s_m[c][g] == -INFINITY) continue;
        const float w = expf(s_m[c][g] - M);
        L = fmaf(s_l[c][g], w, L);
        O = fmaf(s_o[c][g][d], w, O);
      }
    }
    const int64_t row = i * a.n_heads + h0 + g;
    if constexpr (FINAL) {
      a.out[row * D + d] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
      if (d == 0 && a.lse != nullptr) a.lse[row] = L > 0.0f ? M + logf(L) : -INFINITY;
    } else {
      float* w = a.ws + (row * a.splits + split) * (D + 2);
      if (d == 0) {
        w[0] = M;
        w[1] = L;
      }
      w[2 + d] = O;
    }
  }
}

// One CTA (8 warps) per query row (position x head): the splits' (m, l, O)
// combined with weights exp(m_s - M), M the largest m_s.  Warp w takes splits
// w, w + 8, ...: its lanes load O_s as 16-byte (d = 128) or 8-byte (d = 64)
// vectors, all of a warp's loads independent, so the merge runs at L2 latency,
// not one round trip per split.  The eight warp sums are added in warp order:
// deterministic.
constexpr int kMergeWarps = 8;
template <int D>
__global__ void __launch_bounds__(kMergeWarps * 32) attn_merge_kernel(const AttnArgs a) {
  constexpr int EPL = D / 32;  // elements per lane
  __shared__ float s_o[kMergeWarps][D];
  __shared__ float s_l[kMergeWarps];
  __shared__ float s_m[kMergeWarps];
  pdl_trigger();
  pdl_wait();
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int S = a.splits;
  for (int64_t row = blockIdx.x; row < a.s_q * a.n_heads; row += gridDim.x) {
    const float* w = a.ws + row * static_cast<int64_t>(S) * (D + 2);
    float mx = -INFINITY;
    for (int sp = t; sp < S; sp += kMergeWarps * 32) mx = fmaxf(mx, w[static_cast<int64_t>(sp) * (D + 2)]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_m[warp] = mx;
    __syncthreads();
    float M = s_m[0];
#pragma unroll
    for (int i = 1; i < kMergeWarps; ++i) M = fmaxf(M, s_m[i]);
    float o[EPL], L = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
#pragma unroll 4
    for (int sp = warp; sp < S; sp += kMergeWarps) {
      const float* ws = w + static_cast<int64_t>(sp) * (D + 2);
      const float ms = ws[0];
      const float f = (ms == -INFINITY || M == -INFINITY) ? 0.0f : expf(ms - M);
      L = fmaf(ws[1], f, L);
      // O_s starts at an 8-byte boundary (D + 2 floats per split): two float2 per lane for
      // d = 128, one for d = 64
#pragma unroll
      for (int e = 0; e < EPL; e += 2) {
        const float2 v = *reinterpret_cast<const float2*>(ws + 2 + lane * EPL + e);
        o[e] = fmaf(v.x, f, o[e]);
        o[e + 1] = fmaf(v.y, f, o[e + 1]);
      }
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) s_o[warp][lane * EPL + e] = o[e];
    if (lane == 0) s_l[warp] = L;
    __syncthreads();
    if (t < D) {
      float Ot = 0.0f, Lt = 0.0f;
#pragma unroll
      for (int i = 0; i < kMergeWarps; ++i) {
        Ot += s_o[i][t];
        Lt += s_l[i];
      }
      a.out[row * D + t] = __float2half_rn(Lt > 0.0f ? Ot / Lt : 0.0f);
      if (t == 0 && a.lse != nullptr) a.lse[row] = Lt > 0.0f ? M + logf(Lt) : -INFINITY;
    }
    __syncthreads();  // s_o / s_m are reused by the next row
  }
}

// ---------------------------------------------------------------- decode (bulk)
//
// attention_decode with K / V streamed by bulk copies.  The keys of one KV head
// are contiguous ([n_kv_heads][kv_head_stride], key j at j * d), so a CTA's
// split arrives as whole 64-key blocks of K and of V, each ONE cp.async.bulk
// into a two-stage shared-memory ring: all of a block's bytes are in flight at
// once.  Per block the CTA (8 warps, GB query heads of one KV group) forms the
// scores (lane groups of d/8 lanes per key, shuffle-reduced), the block max and
// probabilities per head, and O = alpha * O + P V with one thread per output
// pair of elements -- one rescale per 64 keys, not per key.  The split's
// (m, l, O) goes to the workspace for attn_merge_kernel (split order), or with
// one split straight to out.  Scores use the natural base (expf), like the
// split kernel, so the two share the merge.
constexpr int kDecBlock = 64;  // keys per bulk block

constexpr int kDecWarps = 8;
template <int D, int GB>
struct DecCfg {
  static constexpr int kBlockBytes = kDecBlock * D * 2;  // one block of K (or V)
  static constexpr int kRing = 2;                        // stages at most
  /// Dynamic shared memory for `stages` ring stages plus the barriers.
  static constexpr int smem(int stages) { return stages * 2 * kBlockBytes + 64; }
};

__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int D, int GB, bool FINAL>
__global__ void __launch_bounds__(kDecWarps * 32, 4)
    attn_decode_bulk_kernel(const AttnArgs a, int nst, unsigned int* err,
                            unsigned long long limit_ns) {
  using Cfg = DecCfg<D, GB>;
  constexpr int LPK = D / 8;                 // lanes per key row
  constexpr int KPW = 32 / LPK;              // key rows per warp per step
  constexpr int NP = D / 2;                  // element pairs per head
  constexpr int GS = (kDecWarps * 32) / NP;  // heads one pass of the threads covers
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* ring = dsm;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + nst * 2 * Cfg::kBlockBytes);
  __shared__ float s_p[GB][kDecBlock];
  __shared__ float s_m[GB], s_l[GB], s_alpha[GB];
  __shared__ int s_ok;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % LPK, kgw = lane / LPK;
  const int64_t group = a.n_heads / a.n_kv_heads;
  const int64_t chunks_per_kv = group / GB;
  const int64_t h_kv = blockIdx.y / chunks_per_kv;
  const int64_t h0 = h_kv * group + (blockIdx.y % chunks_per_kv) * GB;
  const int split = blockIdx.x;
  const int64_t j0 = static_cast<int64_t>(split) * a.chunk;
  int64_t j1 = j0 + a.chunk;
  if (j1 > a.s_kv) j1 = a.s_kv;
  const int nblk = j1 > j0 ? static_cast<int>((j1 - j0 + kDecBlock - 1) / kDecBlock) : 0;
  const __half* kh = a.k + h_kv * a.kv_head_stride;
  const __half* vh = a.v + h_kv * a.kv_head_stride;

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
    s_ok = 1;
  }
  if (threadIdx.x < GB) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.0f;
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  // Block b of the split goes to stage b % nst; the use of a stage's barrier
  // by block b is its (b / nst)-th phase.
  auto issue = [&](int b) {  // thread 0
    const int64_t jb = j0 + static_cast<int64_t>(b) * kDecBlock;
    const int64_t n = (j1 - jb < kDecBlock) ? j1 - jb : kDecBlock;
    const uint32_t bytes = static_cast<uint32_t>(n * D * 2);
    uint8_t* st = ring + (b % nst) * 2 * Cfg::kBlockBytes;
    mbar_arrive_expect_tx(&full[b % nst], 2 * bytes);
    bulk_load_1d(st, kh + jb * D, bytes, &full[b % nst]);
    bulk_load_1d(st + Cfg::kBlockBytes, vh + jb * D, bytes, &full[b % nst]);
  };
  int issued = 0;
  if (threadIdx.x == 0) {
    for (; issued < nblk && issued < nst; ++issued) issue(issued);
  }

  float qf[GB][8];
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    load8<true>(a.q + (h0 + g) * D + 8 * sub, qf[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[g][e] *= a.scale;
  }
  const int pr = threadIdx.x % NP;  // this thread's element pair of O
  const int gs = threadIdx.x / NP;  // its heads: gs, gs + GS, ...
  float o0[GB], o1[GB];
#pragma unroll
  for (int g = 0; g < GB; ++g) o0[g] = o1[g] = 0.0f;

  int consumed = 0;
  for (int b = 0; b < nblk; ++b) {
    if (!mbar_wait(&full[b % nst], (b / nst) & 1u, limit_ns, err)) s_ok = 0;
    __syncthreads();
    if (!s_ok) break;
    consumed = b + 1;
    const uint8_t* st = ring + (b % nst) * 2 * Cfg::kBlockBytes;
    const __half* ks = reinterpret_cast<const __half*>(st);
    const __half* vs = reinterpret_cast<const __half*>(st + Cfg::kBlockBytes);
    const int64_t jb = j0 + static_cast<int64_t>(b) * kDecBlock;
    const int n = static_cast<int>((j1 - jb < kDecBlock) ? j1 - jb : kDecBlock);
    // scores: each lane group takes one key per step
    for (int kb = warp * KPW; kb < kDecBlock; kb += kDecWarps * KPW) {
      const int kk = kb + kgw;
      const bool valid = kk < n;
      float kf[8];
      if (valid) {
        const uint4 u = *reinterpret_cast<const uint4*>(ks + kk * D + 8 * sub);
        const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __half22float2(hh[i]);
          kf[2 * i] = t.x;
          kf[2 * i + 1] = t.y;
        }
      }
#pragma unroll
      for (int g = 0; g < GB; ++g) {
        float sc = 0.0f;
        if (valid) {
#pragma unroll
          for (int e = 0; e < 8; ++e) sc = fmaf(qf[g][e], kf[e], sc);
        }
#pragma unroll
        for (int off = LPK / 2; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
        if (sub == 0) s_p[g][kk] = valid ? sc : -INFINITY;
      }
    }
    __syncthreads();
    // per head (warp w takes heads w, w + 4, ...): block max, probabilities, running (m, l)
    for (int g = warp; g < GB; g += kDecWarps) {
      float mx = -INFINITY;
      for (int t = lane; t < kDecBlock; t += 32) mx = fmaxf(mx, s_p[g][t]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = s_m[g];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (int t = lane; t < kDecBlock; t += 32) {
        const float pv = (t < n) ? expf(s_p[g][t] - m_new) : 0.0f;
        s_p[g][t] = pv;
        sum += pv;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      __syncwarp();
      if (lane == 0) {
        const float al = expf(m_old - m_new);  // m_old = -inf: 0
        s_alpha[g] = al;
        s_l[g] = s_l[g] * al + sum;
        s_m[g] = m_new;
      }
    }
    __syncthreads();
    // O = alpha O + P V
#pragma unroll
    for (int g = 0; g < GB; ++g) {
      if (g % GS != gs) continue;
      const float al = s_alpha[g];
      // two interleaved chains per element (even / odd keys), added at the end
      float a0 = 0.0f, a1 = 0.0f, c0 = 0.0f, c1 = 0.0f;
      int t = 0;
#pragma unroll 4
      for (; t + 1 < n; t += 2) {
        const float p0 = s_p[g][t], p1 = s_p[g][t + 1];
        const float2 v0 = __half22float2(reinterpret_cast<const __half2*>(vs + t * D)[pr]);
        const float2 v1 = __half22float2(reinterpret_cast<const __half2*>(vs + (t + 1) * D)[pr]);
        a0 = fmaf(p0, v0.x, a0);
        a1 = fmaf(p0, v0.y, a1);
        c0 = fmaf(p1, v1.x, c0);
        c1 = fmaf(p1, v1.y, c1);
      }
      if (t < n) {
        const float p0 = s_p[g][t];
        const float2 v0 = __half22float2(reinterpret_cast<const __half2*>(vs + t * D)[pr]);
        a0 = fmaf(p0, v0.x, a0);
        a1 = fmaf(p0, v0.y, a1);
      }
      o0[g] = o0[g] * al + (a0 + c0);
      o1[g] = o1[g] * al + (a1 + c1);
    }
    __syncthreads();  // stage b and s_p fully read: refill
    if (threadIdx.x == 0 && issued < nblk) {
      issue(issued);
      ++issued;
    }
  }
  // No copy may be writing shared memory when the CTA leaves (only after a
  // time-out are issued blocks left unconsumed): wait for them, bounded.
  if (threadIdx.x == 0) {
    for (int b = consumed; b < issued; ++b) mbar_wait(&full[b % nst], (b / nst) & 1u, limit_ns, err);
  }
  if (!s_ok) return;
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    if (g % GS != gs) continue;
    const int64_t row = h0 + g;  // one query position
    const float M = s_m[g], L = s_l[g];
    if constexpr (FINAL) {
      const float inv = L > 0.0f ? 1.0f / L : 0.0f;
      reinterpret_cast<__half2*>(a.out + row * D)[pr] = __floats2half2_rn(o0[g] * inv, o1[g] * inv);
      if (pr == 0 && a.lse != nullptr) a.lse[row] = L > 0.0f ? M + logf(L) : -INFINITY;
    } else {
      float* w = a.ws + (row * a.splits + split) * (D + 2);
      if (pr == 0) {
        w[0] = nblk > 0 ? M : -INFINITY;
        w[1] = L;
      }
      w[2 + 2 * pr] = o0[g];
      w[3 + 2 * pr] = o1[g];
    }
  }
}

template <int D, int GB>
int launch_decode_bulk(AttnArgs& a, cudaStream_t st) {
  using Cfg = DecCfg<D, GB>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if ((configured.load() & bit) == 0) {
    B200_CUDA(cudaFuncSetAttribute(attn_decode_bulk_kernel<D, GB, true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::smem(Cfg::kRing)));
    B200_CUDA(cudaFuncSetAttribute(attn_decode_bulk_kernel<D, GB, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cfg::smem(Cfg::kRing)));
    configured.fetch_or(bit);
  }
  const int64_t group = a.n_heads / a.n_kv_heads;
  const dim3 grid(static_cast<unsigned>(a.splits), static_cast<unsigned>(a.n_kv_heads * (group / GB)));
  unsigned int* err = device_error_word();
  const unsigned long long lim = wait_limit_ns();
  // One stage when a split is a single block (more CTAs fit per SM), else two.
  const int nst = a.chunk <= kDecBlock ? 1 : Cfg::kRing;
  const size_t smem = static_cast<size_t>(Cfg::smem(nst));
  if (a.splits == 1) {
    B200_CUDA(launch_pdl(attn_decode_bulk_kernel<D, GB, true>, grid, dim3(kDecWarps * 32), smem,
                         st, a, nst, err, lim));
  } else {
    B200_CUDA(launch_pdl(attn_decode_bulk_kernel<D, GB, false>, grid, dim3(kDecWarps * 32), smem,
                         st, a, nst, err, lim));
    B200_CUDA(launch_pdl(attn_merge_kernel<D>, dim3(static_cast<unsigned>(a.n_heads)),
                         dim3(kMergeWarps * 32), 0, st, a));
  }
  return ENGINE_OK;
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[t] = v;
}

template <int D, int GB, bool VEC>
int launch_split(AttnArgs& a, cudaStream_t st) {
  const int64_t group = a.n_heads / a.n_kv_heads;
  const dim3 grid(static_cast<unsigned>(a.splits),
                  static_cast<unsigned>(a.n_kv_heads * (group / GB)), static_cast<unsigned>(a.s_q));
  if (a.splits == 1) {
    B200_CUDA(launch_pdl(attn_split_kernel<D, GB, VEC, true>, grid, dim3(kAttnWarps * 32), 0, st, a));
  } else {
    B200_CUDA(launch_pdl(attn_split_kernel<D, GB, VEC, false>, grid, dim3(kAttnWarps * 32), 0, st, a));
    const int64_t rows = a.s_q * a.n_heads;
    B200_CUDA(launch_pdl(attn_merge_kernel<D>, dim3(static_cast<unsigned>(rows < 65535 ? rows : 65535)),
                         dim3(kMergeWarps * 32), 0, st, a));
  }
  return ENGINE_OK;
}

template <int D, bool VEC>
int launch_gb(AttnArgs& a, cudaStream_t st) {
  const int64_t group = a.n_heads / a.n_kv_heads;
  if (group % 4 == 0) return launch_split<D, 4, VEC>(a, st);
  if (group % 2 == 0) return launch_split<D, 2, VEC>(a, st);
  return launch_split<D, 1, VEC>(a, st);
}

// Shared body of both entry points (arguments already validated).
int run_attention(const __half* q, const __half* k, const __half* v, __half* out, int64_t s_q,
                  int64_t s_kv, int64_t n_heads, int64_t n_kv_heads, int64_t d, int64_t stride,
                  float scale, int64_t q_pos_offset, bool causal, float* lse, int split_kv,
                  cudaStream_t st, const char* what) {
  if (s_q == 0) return ENGINE_OK;
  if (s_kv == 0) {
    B200_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(s_q * n_heads * d) * 2, st));
    if (lse != nullptr) {
      fill_kernel<<<static_cast<unsigned>((s_q * n_heads + 255) / 256), 256, 0, st>>>(
          lse, s_q * n_heads, -INFINITY);
    }
    return check_launch(what);
  }
  AttnArgs a{q, k, v, out, lse, nullptr, s_q, s_kv, n_heads, n_kv_heads, stride, q_pos_offset,
             scale, causal ? 1 : 0, 1, s_kv};
  const int64_t group = n_heads / n_kv_heads;
  const int64_t gb = group % 4 == 0 ? 4 : (group % 2 == 0 ? 2 : 1);
  const int64_t ctas = s_q * n_kv_heads * (group / gb);
  const bool bulk = s_q == 1 && !causal && stride % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                      reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) % 16) == 0;
  static const int dec_tc_env = env_flag("ENGINE_ATTN_DECODE_TC", 1);
  if (bulk && split_kv <= 0 && dec_tc_env != 0) {
    // tcgen05 decode (attention_tc.cu), its splits merged inside one cluster per
    // KV head; shapes it does not take fall through to the bulk kernel.
    int64_t chunk = 0;
    const int sp = attention_decode_tc_splits(s_kv, n_kv_heads, &chunk);
    float* wst = nullptr;
    if (sp > 1) {
      const size_t bytes = static_cast<size_t>(n_heads) * sp * (d + 2) * sizeof(float);
      wst = static_cast<float*>(scratch_alloc(bytes, st));
      if (wst == nullptr)
        return set_error(ENGINE_ERR_CUDA, std::string(what) + ": workspace allocation failed");
    }
    int rc = attention_decode_tc(q, k, v, out, lse, wst, s_kv, n_heads, n_kv_heads, d, stride,
                                 scale, st);
    if (rc == ENGINE_OK && sp > 1) {
      a.ws = wst;
      a.splits = sp;
      a.chunk = chunk;
      const cudaError_t e = launch_pdl(attn_merge_kernel<128>, dim3(static_cast<unsigned>(n_heads)),
                                       dim3(kMergeWarps * 32), 0, st, a);
      if (e != cudaSuccess) rc = set_cuda_error(e, "attn_merge_kernel");
      else rc = check_launch(what);
    }
    if (wst != nullptr) scratch_free(wst, st);
    if (rc != ENGINE_ERR_UNSUPPORTED) return rc;
  }
  int64_t splits = split_kv;
  if (splits <= 0 && bulk) {
    // decode: at least about four CTAs per SM, each split a whole number of
    // 64-key blocks (one block when the keys allow)
    const int64_t want = (4 * static_cast<int64_t>(sm_count()) + ctas - 1) / ctas;
    int64_t chunk = (s_kv + want - 1) / want;
    chunk = (chunk + kDecBlock - 1) / kDecBlock * kDecBlock;
    splits = (s_kv + chunk - 1) / chunk;
  } else if (splits <= 0) {  // enough CTAs for two per SM, each split at least 128 keys
    const int64_t want = (2 * static_cast<int64_t>(sm_count()) + ctas - 1) / ctas;
    const int64_t most = (s_kv + 127) / 128;
    splits = want < most ? want : most;
    if (splits < 1) splits = 1;
  }
  if (splits > s_kv) splits = s_kv;
  if (splits > 65535) splits = 65535;
  a.chunk = (s_kv + splits - 1) / splits;
  a.splits = static_cast<int>((s_kv + a.chunk - 1) / a.chunk);
  float* ws = nullptr;
  if (a.splits > 1) {
    const size_t bytes = static_cast<size_t>(s_q * n_heads) * a.splits * (d + 2) * sizeof(float);
    ws = static_cast<float*>(scratch_alloc(bytes, st));
    if (ws == nullptr) return set_error(ENGINE_ERR_CUDA, std::string(what) + ": workspace allocation failed");
    a.ws = ws;
  }
  const bool vec = (reinterpret_cast<uintptr_t>(q) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(k) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(v) % 16 == 0) && (stride % 8 == 0);
  int rc;
  if (bulk) {
    if (d == 64) {
      rc = gb == 4 ? launch_decode_bulk<64, 4>(a, st)
                   : (gb == 2 ? launch_decode_bulk<64, 2>(a, st) : launch_decode_bulk<64, 1>(a, st));
    } else {
      rc = gb == 4 ? launch_decode_bulk<128, 4>(a, st)
                   : (gb == 2 ? launch_decode_bulk<128, 2>(a, st) : launch_decode_bulk<128, 1>(a, st));
    }
  } else if (d == 64) {
    rc = vec ? launch_gb<64, true>(a, st) : launch_gb<64, false>(a, st);
  } else {
    rc = vec ? launch_gb<128, true>(a, st) : launch_gb<128, false>(a, st);
  }
  if (ws != nullptr) scratch_free(ws, st);
  if (rc != ENGINE_OK) return rc;
  return check_launch(what);
}

// ---------------------------------------------------------------- KV cache write
//
// Scatters token-major K / V rows into head-major caches (the engine's
// kv_cache_write, kernels.hpp:184; kernels/attention_bridge.cu:87), for
// n_seq sequences of s_new tokens each: source row r = b * s_new + t holds
// K[b, t] at k_new + r * row_pitch as [n_kv_heads][head_dim] (row_pitch = the
// row length for the engine's contiguous form; the Q/K/V projection's output
// row for the fused form), and lands at
// cache[((b * n_kv_heads + h) * kv_max_seq_len + pos_offset + t) * head_dim].
// One thread per 16 bytes when everything is 16-byte aligned, else per element;
// a pure copy (bit-exact).
template <bool VEC>
__global__ void kv_cache_write_kernel(const __half* __restrict__ k_new,
                                      const __half* __restrict__ v_new, int64_t row_pitch,
                                      __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                      int64_t n_seq, int64_t s_new, int64_t n_kv_heads,
                                      int64_t head_dim, int64_t pos_offset, int64_t max_len) {
  pdl_trigger();
  pdl_wait();
  constexpr int W = VEC ? 8 : 1;  // halves per thread
  const int64_t per_row = n_kv_heads * head_dim / W;
  const int64_t total = n_seq * s_new * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row;  // source row = b * s_new + t
    const int64_t c = (i - r * per_row) * W;  // element within the row
    const int64_t h = c / head_dim, e = c - h * head_dim;
    const int64_t b = r / s_new, t = r - b * s_new;
    const int64_t dst = ((b * n_kv_heads + h) * max_len + pos_offset + t) * head_dim + e;
    const int64_t src = r * row_pitch + c;
    if constexpr (VEC) {
      *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(k_new + src);
      *reinterpret_cast<uint4*>(v_cache + dst) = *reinterpret_cast<const uint4*>(v_new + src);
    } else {
      k_cache[dst] = k_new[src];
      v_cache[dst] = v_new[src];
    }
  }
}

int kv_cache_write_impl(const __half* k_new, const __half* v_new, int64_t row_pitch,
                        __half* k_cache, __half* v_cache, int64_t n_seq, int64_t s_new,
                        int64_t n_kv_heads, int64_t head_dim, int64_t pos_offset, int64_t max_len,
                        cudaStream_t st) {
  const bool vec = head_dim % 8 == 0 && row_pitch % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
                     reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) %
                    16) == 0;
  const int64_t units = n_seq * s_new * n_kv_heads * head_dim / (vec ? 8 : 1);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  const int64_t blocks = (units + 255) / 256;
  const unsigned grid = static_cast<unsigned>(blocks < cap ? blocks : cap);
  if (vec) {
    B200_CUDA(launch_pdl(kv_cache_write_kernel<true>, dim3(grid), dim3(256), 0, st, k_new, v_new,
                         row_pitch, k_cache, v_cache, n_seq, s_new, n_kv_heads, head_dim,
                         pos_offset, max_len));
  } else {
    B200_CUDA(launch_pdl(kv_cache_write_kernel<false>, dim3(grid), dim3(256), 0, st, k_new, v_new,
                         row_pitch, k_cache, v_cache, n_seq, s_new, n_kv_heads, head_dim,
                         pos_offset, max_len));
  }
  return check_launch("kv_cache_write");
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int engine_cuda_attention_prefill(const engine_half_t* q, const engine_half_t* k,
                                  const engine_half_t* v, engine_half_t* out, int64_t s_q,
                                  int64_t s_kv, int64_t n_heads, int64_t n_kv_heads,
                                  int64_t head_dim, int64_t kv_head_stride, float scale,
                                  int64_t q_pos_offset, int is_causal, float* out_lse,
                                  engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(q != nullptr, "attention_prefill: q is null");
  B200_REQUIRE(k != nullptr, "attention_prefill: k is null");
  B200_REQUIRE(v != nullptr, "attention_prefill: v is null");
  B200_REQUIRE(out != nullptr, "attention_prefill: out is null");
  B200_REQUIRE(s_q >= 0, "attention_prefill: s_q must be non-negative");
  B200_REQUIRE(s_kv >= 0, "attention_prefill: s_kv must be non-negative");
  B200_REQUIRE(q_pos_offset >= 0, "attention_prefill: q_pos_offset must be non-negative");
  B200_REQUIRE(n_heads > 0, "attention_prefill: n_heads must be positive");
  B200_REQUIRE(n_kv_heads > 0, "attention_prefill: n_kv_heads must be positive");
  B200_REQUIRE(n_heads % n_kv_heads == 0,
               "attention_prefill: n_heads must be divisible by n_kv_heads");
  B200_REQUIRE(head_dim == 64 || head_dim == 128,
               "attention_prefill: head_dim must be 64 or 128");
  B200_REQUIRE(std::isfinite(scale), "attention_prefill: scale must be finite");
  B200_REQUIRE(kv_head_stride >= (s_kv > 0 ? s_kv * head_dim : 0),
               "attention_prefill: kv_head_stride < s_kv * head_dim");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static const int tc_env = env_flag("ENGINE_ATTN_TC", 1);
  if (tc_env != 0 && s_q >= kAttnTcMinRows && s_kv > 0) {
    // tcgen05 FlashAttention (attention_tc.cu); shapes or alignments it does not
    // take fall through to the CUDA-core kernel below.
    const int rc = attention_prefill_tc(
        reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
        reinterpret_cast<const __half*>(v), reinterpret_cast<__half*>(out), s_q, s_kv, n_heads,
        n_kv_heads, head_dim, kv_head_stride, scale, q_pos_offset, is_causal != 0, out_lse, st);
    if (rc != ENGINE_ERR_UNSUPPORTED) return rc;
  }
  B200_REQUIRE(s_q <= 65535 && n_heads <= 65535, "attention_prefill: s_q or n_heads too large");
  return run_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                       reinterpret_cast<const __half*>(v), reinterpret_cast<__half*>(out), s_q,
                       s_kv, n_heads, n_kv_heads, head_dim, kv_head_stride, scale, q_pos_offset,
                       is_causal != 0, out_lse, 0, static_cast<cudaStream_t>(stream),
                       "attention_prefill");
  B200_ENTRY_END
}

int engine_cuda_attention_decode(const engine_half_t* q, const engine_half_t* k,
                                 const engine_half_t* v, engine_half_t* out, int64_t kv_len,
                                 int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                                 int64_t kv_head_stride, float scale, int split_kv,
                                 engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(q != nullptr, "attention_decode: q is null");
  B200_REQUIRE(k != nullptr, "attention_decode: k is null");
  B200_REQUIRE(v != nullptr, "attention_decode: v is null");
  B200_REQUIRE(out != nullptr, "attention_decode: out is null");
  B200_REQUIRE(kv_len >= 0, "attention_decode: kv_len must be non-negative");
  B200_REQUIRE(n_heads > 0, "attention_decode: n_heads must be positive");
  B200_REQUIRE(n_kv_heads > 0, "attention_decode: n_kv_heads must be positive");
  B200_REQUIRE(n_heads % n_kv_heads == 0,
               "attention_decode: n_heads must be divisible by n_kv_heads");
  B200_REQUIRE(head_dim == 64 || head_dim == 128,
               "attention_decode: head_dim must be 64 or 128");
  B200_REQUIRE(std::isfinite(scale), "attention_decode: scale must be finite");
  B200_REQUIRE(split_kv >= 0, "attention_decode: split_kv must be non-negative");
  B200_REQUIRE(kv_head_stride >= (kv_len > 0 ? kv_len * head_dim : 0),
               "attention_decode: kv_head_stride < kv_len * head_dim");
  B200_REQUIRE(n_heads <= 65535, "attention_decode: n_heads too large");
  return run_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                       reinterpret_cast<const __half*>(v), reinterpret_cast<__half*>(out), 1,
                       kv_len, n_heads, n_kv_heads, head_dim, kv_head_stride, scale, 0, false,
                       nullptr, split_kv, static_cast<cudaStream_t>(stream), "attention_decode");
  B200_ENTRY_END
}

int engine_cuda_kv_cache_write(const engine_half_t* k_new, const engine_half_t* v_new,
                               engine_half_t* k_cache, engine_half_t* v_cache, int64_t s_new,
                               int64_t n_kv_heads, int64_t head_dim, int64_t pos_offset,
                               int64_t kv_max_seq_len, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  // The engine's checks and messages (kernels/attention_bridge.cu:89-103).
  B200_REQUIRE(s_new >= 0, "kv_cache_write: s_new must be non-negative");
  B200_REQUIRE(n_kv_heads > 0, "kv_cache_write: n_kv_heads must be positive");
  B200_REQUIRE(head_dim > 0, "kv_cache_write: head_dim must be positive");
  B200_REQUIRE(pos_offset >= 0, "kv_cache_write: pos_offset must be non-negative");
  B200_REQUIRE(kv_max_seq_len >= pos_offset + s_new,
               "kv_cache_write: kv_max_seq_len < pos_offset + s_new");
  if (s_new == 0) return ENGINE_OK;
  B200_REQUIRE(k_new != nullptr && v_new != nullptr, "kv_cache_write: k_new/v_new is null");
  B200_REQUIRE(k_cache != nullptr && v_cache != nullptr, "kv_cache_write: k_cache/v_cache is null");
  return kv_cache_write_impl(reinterpret_cast<const __half*>(k_new),
                             reinterpret_cast<const __half*>(v_new), n_kv_heads * head_dim,
                             reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache),
                             1, s_new, n_kv_heads, head_dim, pos_offset, kv_max_seq_len,
                             static_cast<cudaStream_t>(stream));
  B200_ENTRY_END
}

int engine_cuda_kv_cache_write_rows(const engine_half_t* k_new, const engine_half_t* v_new,
                                    int64_t row_pitch, engine_half_t* k_cache,
                                    engine_half_t* v_cache, int64_t n_seq, int64_t s_new,
                                    int64_t n_kv_heads, int64_t head_dim, int64_t pos_offset,
                                    int64_t kv_max_seq_len, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(n_seq >= 0, "kv_cache_write_rows: n_seq must be non-negative");
  B200_REQUIRE(s_new >= 0, "kv_cache_write_rows: s_new must be non-negative");
  B200_REQUIRE(n_kv_heads > 0, "kv_cache_write_rows: n_kv_heads must be positive");
  B200_REQUIRE(head_dim > 0, "kv_cache_write_rows: head_dim must be positive");
  B200_REQUIRE(row_pitch >= n_kv_heads * head_dim,
               "kv_cache_write_rows: row_pitch < n_kv_heads * head_dim");
  B200_REQUIRE(pos_offset >= 0, "kv_cache_write_rows: pos_offset must be non-negative");
  B200_REQUIRE(kv_max_seq_len >= pos_offset + s_new,
               "kv_cache_write_rows: kv_max_seq_len < pos_offset + s_new");
  if (s_new == 0 || n_seq == 0) return ENGINE_OK;
  B200_REQUIRE(k_new != nullptr && v_new != nullptr, "kv_cache_write_rows: k_new/v_new is null");
  B200_REQUIRE(k_cache != nullptr && v_cache != nullptr,
               "kv_cache_write_rows: k_cache/v_cache is null");
  return kv_cache_write_impl(reinterpret_cast<const __half*>(k_new),
                             reinterpret_cast<const __half*>(v_new), row_pitch,
                             reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache),
                             n_seq, s_new, n_kv_heads, head_dim, pos_offset, kv_max_seq_len,
                             static_cast<cudaStream_t>(stream));
  B200_ENTRY_END
}

}  // extern "C"
